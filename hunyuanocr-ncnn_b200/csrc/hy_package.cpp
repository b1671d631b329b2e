// Model-package reader: the ncnn param/bin files that the reference's exporter
// writes (export/export_text_embed.py, export/export_text_decoder_kv.py with
// export/add_kvcache.py, export/dflash_export.py; pnnx with fp16=0, optlevel=2,
// export/_common.py:80-98) read into the library's weight structs.
//
// The reference loads the same files into ncnn::Net through a memory-mapped
// DataReader (src/mapped_model_file.cpp:156 mmap, :375 load_shared_model_data),
// one mapping of text_embed.ncnn.bin serving both the embedding and the tied LM
// head (src/text_runtime.cpp:1705-1745). Here the .bin files are mapped the
// same way and the weights go to the device once (hy_ctx_create copies the tied
// table once and uses it for both).
//
// ncnn's model-bin layout, as its layers read it (restated, ncnn @ dda2e28 is
// not vendored): every weight-bearing layer, in .param order, reads its arrays
// from the .bin one after the other. An array read with "type 0" starts with a
// 4-byte tag: 0 or 0x0002C056 = raw fp32 follows, 0x01306B47 = fp16 follows
// (padded to 4 bytes), 0x000D4B38 = int8 (not used by this model), anything
// else = an 8-bit table quantisation (not used). "Type 1" arrays are raw fp32
// without a tag. The arrays per layer type:
//   Gemm         constantA: A (M x K or K x M), constantB: B (transB ? N rows
//                of K : K rows of N), constantC (broadcast type != -1): C, all
//                type 0
//   InnerProduct weight (weight_data_size, type 0), bias (num_output, type 1)
//   Embed        weight (weight_data_size = input_dim x num_output, type 0),
//                bias (num_output, type 1)
//   RMSNorm      gamma (affine_size, type 1) when affine
//   LayerNorm    gamma, beta (affine_size each, type 1) when affine
//   MemoryData   w x h x d x c values of load_type (default 1)
// Every other layer type carries no weights; the reader checks that it ends
// exactly at the end of the .bin, which catches any layer it does not know.
//
// Names: pnnx names a module's layer by its path in the traced wrapper
// (layers.<i>.self_attn.q_proj, layers.<i>.mlp.down_proj, norm, fc, ...), and
// a folded parameter by its path too (layers.<i>.input_layernorm.weight).
#include "hy_decode.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

namespace hy_internal {
void set_last_error(const std::string& msg);   // hy_capi.cu: the message hy_last_error returns
}

namespace {

int perr(int status, const std::string& msg)
{
    hy_internal::set_last_error(msg);
    return status;
}

// Read-only private mapping of a whole file.
class Mapping {
public:
    ~Mapping()
    {
        if (data_) munmap(const_cast<unsigned char*>(data_), size_);
    }
    int open(const std::string& path)
    {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) return perr(HY_ERR_INVALID_ARGUMENT, "failed to open model file: " + path + " (" + std::strerror(errno) + ")");
        struct stat st{};
        if (fstat(fd, &st) != 0 || st.st_size <= 0)
        {
            ::close(fd);
            return perr(HY_ERR_INVALID_ARGUMENT, "model file is empty or too large to map: " + path);
        }
        void* v = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (v == MAP_FAILED)
            return perr(HY_ERR_INVALID_ARGUMENT, "failed to map model file: " + path + " (" + std::strerror(errno) + ")");
        data_ = static_cast<const unsigned char*>(v);
        size_ = static_cast<size_t>(st.st_size);
        return HY_OK;
    }
    const unsigned char* data() const { return data_; }
    size_t size() const { return size_; }

private:
    const unsigned char* data_ = nullptr;
    size_t size_ = 0;
};

struct ParamLayer {
    std::string type, name;
    std::map<int, std::string> params;
    int geti(int key, int dflt) const
    {
        auto it = params.find(key);
        return it == params.end() ? dflt : std::atoi(it->second.c_str());
    }
};

int parse_param(const std::string& path, std::vector<ParamLayer>* layers)
{
    std::ifstream f(path);
    if (!f) return perr(HY_ERR_INVALID_ARGUMENT, "failed to open model param: " + path);
    std::string line;
    if (!std::getline(f, line) || line.find("7767517") != 0) return perr(HY_ERR_INVALID_ARGUMENT, "not an ncnn param file: " + path);
    int n_layers = 0, n_blobs = 0;
    if (!std::getline(f, line) || std::sscanf(line.c_str(), "%d %d", &n_layers, &n_blobs) != 2 || n_layers < 0)
        return perr(HY_ERR_INVALID_ARGUMENT, "bad layer / blob count line in " + path);
    while (std::getline(f, line))
    {
        std::istringstream ss(line);
        ParamLayer l;
        int nin = 0, nout = 0;
        if (!(ss >> l.type)) continue;   // blank line
        if (!(ss >> l.name >> nin >> nout) || nin < 0 || nout < 0)
            return perr(HY_ERR_INVALID_ARGUMENT, "bad layer line in " + path + ": " + line);
        std::string tok;
        for (int i = 0; i < nin + nout; ++i)
            if (!(ss >> tok)) return perr(HY_ERR_INVALID_ARGUMENT, "missing blob names in " + path + ": " + line);
        while (ss >> tok)
        {
            const size_t eq = tok.find('=');
            if (eq == std::string::npos) return perr(HY_ERR_INVALID_ARGUMENT, "bad parameter '" + tok + "' in " + path);
            l.params[std::atoi(tok.substr(0, eq).c_str())] = tok.substr(eq + 1);   // arrays (key <= -23300) kept raw
        }
        layers->push_back(std::move(l));
    }
    if (static_cast<int>(layers->size()) != n_layers)
        return perr(HY_ERR_INVALID_ARGUMENT, path + " declares " + std::to_string(n_layers) + " layers but lists " +
                                                 std::to_string(layers->size()));
    return HY_OK;
}

// IEEE binary16 -> binary32 (exact; subnormals normalised).
float half_to_float(uint16_t h)
{
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0)
    {
        if (man == 0) bits = sign;
        else
        {
            exp = 113;   // 127 - 15 + 1
            while (!(man & 0x400u))
            {
                man <<= 1;
                --exp;
            }
            bits = sign | (exp << 23) | ((man & 0x3FFu) << 13);
        }
    }
    else if (exp == 31) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// One weight array read from a .bin: fp32 in place (pointer into the mapping)
// or converted from fp16 into `owned`.
struct Array {
    const float* data = nullptr;
    size_t count = 0;
    std::shared_ptr<std::vector<float>> owned;
};

class BinReader {
public:
    BinReader(const Mapping& m, const std::string& path) : m_(m), path_(path) {}
    int load(size_t count, int type, Array* out)
    {
        uint32_t tag = 0;
        if (type == 0)
        {
            if ((rc_ = need(4))) return rc_;
            std::memcpy(&tag, m_.data() + off_, 4);
            off_ += 4;
        }
        out->count = count;
        if (type == 1 || tag == 0 || tag == 0x0002C056u)
        {
            if ((rc_ = need(count * 4))) return rc_;
            if ((reinterpret_cast<uintptr_t>(m_.data() + off_) & 3u) != 0)
                return perr(HY_ERR_INVALID_ARGUMENT, path_ + ": fp32 array at an unaligned offset");
            out->data = reinterpret_cast<const float*>(m_.data() + off_);
            off_ += count * 4;
            return HY_OK;
        }
        if (tag == 0x01306B47u)
        {
            const size_t bytes = (count * 2 + 3) / 4 * 4;
            if ((rc_ = need(bytes))) return rc_;
            auto v = std::make_shared<std::vector<float>>(count);
            const unsigned char* p = m_.data() + off_;
            for (size_t i = 0; i < count; ++i)
            {
                uint16_t h;
                std::memcpy(&h, p + 2 * i, 2);
                (*v)[i] = half_to_float(h);
            }
            off_ += bytes;
            out->owned = v;
            out->data = v->data();
            return HY_OK;
        }
        return perr(HY_ERR_UNSUPPORTED, path_ + ": weight array with storage tag 0x" + hex(tag) + " at offset " +
                                            std::to_string(off_ - 4) + " (only fp32 and fp16 weights are supported)");
    }
    size_t offset() const { return off_; }

private:
    int need(size_t bytes)
    {
        if (off_ > m_.size() || bytes > m_.size() - off_)
            return perr(HY_ERR_INVALID_ARGUMENT, path_ + ": model bin is shorter than its param file describes (needs " +
                                                     std::to_string(off_ + bytes) + " bytes, has " +
                                                     std::to_string(m_.size()) + ")");
        return HY_OK;
    }
    static std::string hex(uint32_t v)
    {
        char b[16];
        std::snprintf(b, sizeof b, "%08X", v);
        return b;
    }
    const Mapping& m_;
    std::string path_;
    size_t off_ = 0;
    int rc_ = HY_OK;
};

// A named weight of the package: rows x cols (cols = 1 for vectors).
struct Weight {
    Array a;
    int rows = 0, cols = 0;
    std::string layer;   // the layer that held it (messages)
};

// Walk a param/bin pair and collect every weight by layer name.
int read_weights(const std::string& param, const std::string& bin, const Mapping& m,
                 std::vector<std::pair<std::string, Weight>>* out)
{
    std::vector<ParamLayer> layers;
    int rc = parse_param(param, &layers);
    if (rc) return rc;
    BinReader r(m, bin);
    auto add = [&](const ParamLayer& l, const Array& a, int rows, int cols) {
        Weight w;
        w.a = a;
        w.rows = rows;
        w.cols = cols;
        w.layer = l.type + " " + l.name;
        out->emplace_back(l.name, w);
    };
    for (const ParamLayer& l : layers)
    {
        Array a;
        if (l.type == "Gemm")
        {
            const int transA = l.geti(2, 0), transB = l.geti(3, 0), cA = l.geti(4, 0), cB = l.geti(5, 0),
                      cC = l.geti(6, 0), M = l.geti(7, 0), N = l.geti(8, 0), K = l.geti(9, 0), bC = l.geti(10, 0);
            if (l.geti(18, 0) != 0) return perr(HY_ERR_UNSUPPORTED, "int8 Gemm " + l.name + " is not supported");
            (void)transA;
            if (cA && (rc = r.load(static_cast<size_t>(M) * K, 0, &a))) return rc;
            if (cB)
            {
                if (N <= 0 || K <= 0) return perr(HY_ERR_INVALID_ARGUMENT, "Gemm " + l.name + " has constant B without N / K");
                if ((rc = r.load(static_cast<size_t>(N) * K, 0, &a))) return rc;
                if (!transB) return perr(HY_ERR_UNSUPPORTED, "Gemm " + l.name + " stores B untransposed (K x N)");
                add(l, a, N, K);   // nn.Linear layout [out x in]
            }
            if (cC && bC != -1)
            {
                const size_t n = (bC == 0) ? 1 : (bC == 1 || bC == 2) ? static_cast<size_t>(M)
                                 : (bC == 3) ? static_cast<size_t>(M) * N : static_cast<size_t>(N);
                if ((rc = r.load(n, 0, &a))) return rc;
                return perr(HY_ERR_UNSUPPORTED, "Gemm " + l.name + " has a bias, which this model does not");
            }
        }
        else if (l.type == "InnerProduct")
        {
            const int nout = l.geti(0, 0), bias = l.geti(1, 0), wsize = l.geti(2, 0);
            if (l.geti(8, 0) != 0) return perr(HY_ERR_UNSUPPORTED, "int8 InnerProduct " + l.name + " is not supported");
            if (nout <= 0 || wsize <= 0 || wsize % nout) return perr(HY_ERR_INVALID_ARGUMENT, "bad InnerProduct " + l.name);
            if ((rc = r.load(static_cast<size_t>(wsize), 0, &a))) return rc;
            add(l, a, nout, wsize / nout);
            if (bias) return perr(HY_ERR_UNSUPPORTED, "InnerProduct " + l.name + " has a bias, which this model does not");
        }
        else if (l.type == "Embed")
        {
            const int nout = l.geti(0, 0), in_dim = l.geti(1, 0), bias = l.geti(2, 0), wsize = l.geti(3, 0);
            if (l.geti(18, 0) != 0) return perr(HY_ERR_UNSUPPORTED, "int8 Embed " + l.name + " is not supported");
            if (nout <= 0 || in_dim <= 0 || static_cast<long long>(wsize) != static_cast<long long>(nout) * in_dim)
                return perr(HY_ERR_INVALID_ARGUMENT, "bad Embed " + l.name);
            if ((rc = r.load(static_cast<size_t>(wsize), 0, &a))) return rc;
            add(l, a, in_dim, nout);
            if (bias) return perr(HY_ERR_UNSUPPORTED, "Embed " + l.name + " has a bias, which this model does not");
        }
        else if (l.type == "RMSNorm" || l.type == "LayerNorm")
        {
            const int n = l.geti(0, 0), affine = l.geti(2, 1);
            if (!affine) continue;
            if ((rc = r.load(static_cast<size_t>(n), 1, &a))) return rc;
            add(l, a, n, 1);
            if (l.type == "LayerNorm")
            {
                Array beta;
                if ((rc = r.load(static_cast<size_t>(n), 1, &beta))) return rc;
            }
        }
        else if (l.type == "MemoryData")
        {
            const int w = l.geti(0, 0), h = l.geti(1, 0), d = l.geti(11, 0), c = l.geti(2, 0), type = l.geti(21, 1);
            const size_t n = static_cast<size_t>(w ? w : 1) * (h ? h : 1) * (d ? d : 1) * (c ? c : 1);
            if ((rc = r.load(n, type, &a))) return rc;
            // A 2-D constant is [h rows x w columns] (a Linear weight as pnnx folds it: [out x in]).
            add(l, a, h ? h : static_cast<int>(n), h ? w : 1);
        }
    }
    if (r.offset() != m.size())
        return perr(HY_ERR_INVALID_ARGUMENT, bin + ": " + std::to_string(m.size() - r.offset()) +
                                                 " bytes left after the last weight of " + param +
                                                 " (a weighted layer type this reader does not know, or a mismatched pair)");
    return HY_OK;
}

// The slot a layer name stands for: (layer index or -1, field), or false.
bool slot_of(const std::string& name, int* layer, std::string* field)
{
    static const char* kFields[][2] = {
        {".self_attn.q_proj", "q_proj"},         {".self_attn.k_proj", "k_proj"},
        {".self_attn.v_proj", "v_proj"},         {".self_attn.o_proj", "o_proj"},
        {".self_attn.query_layernorm", "query_norm"}, {".self_attn.key_layernorm", "key_norm"},
        {".self_attn.q_norm", "query_norm"},     {".self_attn.k_norm", "key_norm"},
        {".post_attention_layernorm", "post_norm"}, {".input_layernorm", "input_norm"},
        {".mlp.gate_proj", "gate_proj"},         {".mlp.up_proj", "up_proj"},
        {".mlp.down_proj", "down_proj"},
    };
    const size_t p = name.find("layers.");
    if (p != std::string::npos)
    {
        size_t q = p + 7;
        if (q >= name.size() || !std::isdigit(static_cast<unsigned char>(name[q]))) return false;
        int idx = 0;
        while (q < name.size() && std::isdigit(static_cast<unsigned char>(name[q]))) idx = idx * 10 + (name[q++] - '0');
        const std::string rest = name.substr(q);
        for (auto& f : kFields)
        {
            const size_t flen = std::strlen(f[0]);
            // The field path, then nothing, ".weight", or a pnnx duplicate suffix ("_1").
            if (rest.compare(0, flen, f[0]) == 0)
            {
                const std::string tail = rest.substr(flen);
                if (tail.empty() || tail == ".weight" || (tail[0] == '_' && tail.find('.') == std::string::npos))
                {
                    *layer = idx;
                    *field = f[1];
                    return true;
                }
            }
        }
        return false;
    }
    std::string base = name;
    if (base.size() > 7 && base.compare(base.size() - 7, 7, ".weight") == 0) base = base.substr(0, base.size() - 7);
    const size_t dot = base.rfind('.');
    const std::string last = (dot == std::string::npos) ? base : base.substr(dot + 1);
    if (last == "norm" || last == "hidden_norm" || last == "fc" || last == "embed_tokens")
    {
        *layer = -1;
        *field = last;
        return true;
    }
    return false;
}

// The weights of one network by slot; duplicates (a module called twice) must agree.
struct Slots {
    std::map<std::pair<int, std::string>, Weight> w;
    int max_layer = -1;
};

int collect(const std::vector<std::pair<std::string, Weight>>& named, Slots* s)
{
    for (const auto& nw : named)
    {
        int layer = -1;
        std::string field;
        if (!slot_of(nw.first, &layer, &field)) continue;   // a constant this path does not use
        const auto key = std::make_pair(layer, field);
        auto it = s->w.find(key);
        if (it != s->w.end())
        {
            const Weight& o = it->second;
            if (o.a.count != nw.second.a.count || std::memcmp(o.a.data, nw.second.a.data, o.a.count * 4) != 0)
                return perr(HY_ERR_INVALID_ARGUMENT, "layers " + o.layer + " and " + nw.second.layer +
                                                         " hold different weights for the same module");
            continue;
        }
        s->w[key] = nw.second;
        if (layer > s->max_layer) s->max_layer = layer;
    }
    return HY_OK;
}

int need(const Slots& s, int layer, const char* field, int rows, int cols, const std::string& what, const float** out)
{
    auto it = s.w.find(std::make_pair(layer, std::string(field)));
    const std::string where = (layer >= 0 ? "layers." + std::to_string(layer) + "." : std::string()) + field;
    if (it == s.w.end()) return perr(HY_ERR_INVALID_ARGUMENT, what + ": no weight for " + where);
    const Weight& w = it->second;
    if (w.rows != rows || w.cols != cols || w.a.count != static_cast<size_t>(rows) * cols)
        return perr(HY_ERR_INVALID_ARGUMENT, what + ": " + where + " (" + w.layer + ") holds " + std::to_string(w.rows) +
                                                 " x " + std::to_string(w.cols) + ", expected " + std::to_string(rows) +
                                                 " x " + std::to_string(cols));
    *out = w.a.data;
    return HY_OK;
}

// Everything a loaded package keeps alive while its weights are uploaded.
struct Package {
    Mapping embed_bin, decoder_bin, draft_bin;
    Slots embed, decoder, draft;
    int vocab = 0, layers = 0, ffn = 0, draft_layers = 0;
    std::vector<hy_layer_weights> lw, dlw;
    hy_weights w{};
    hy_draft_weights dw{};
};

int layer_weights(const Slots& s, int l, int ffn, const std::string& what, hy_layer_weights* o)
{
    int rc;
    if ((rc = need(s, l, "input_norm", HY_HIDDEN, 1, what, &o->input_norm))) return rc;
    if ((rc = need(s, l, "q_proj", HY_NUM_Q_HEADS * HY_HEAD_DIM, HY_HIDDEN, what, &o->q_proj))) return rc;
    if ((rc = need(s, l, "k_proj", HY_NUM_KV_HEADS * HY_HEAD_DIM, HY_HIDDEN, what, &o->k_proj))) return rc;
    if ((rc = need(s, l, "v_proj", HY_NUM_KV_HEADS * HY_HEAD_DIM, HY_HIDDEN, what, &o->v_proj))) return rc;
    if ((rc = need(s, l, "query_norm", HY_HEAD_DIM, 1, what, &o->query_norm))) return rc;
    if ((rc = need(s, l, "key_norm", HY_HEAD_DIM, 1, what, &o->key_norm))) return rc;
    if ((rc = need(s, l, "o_proj", HY_HIDDEN, HY_NUM_Q_HEADS * HY_HEAD_DIM, what, &o->o_proj))) return rc;
    if ((rc = need(s, l, "post_norm", HY_HIDDEN, 1, what, &o->post_norm))) return rc;
    if ((rc = need(s, l, "gate_proj", ffn, HY_HIDDEN, what, &o->gate_proj))) return rc;
    if ((rc = need(s, l, "up_proj", ffn, HY_HIDDEN, what, &o->up_proj))) return rc;
    return need(s, l, "down_proj", HY_HIDDEN, ffn, what, &o->down_proj);
}

int ffn_of(const Slots& s, const std::string& what, int* ffn)
{
    auto it = s.w.find(std::make_pair(0, std::string("gate_proj")));
    if (it == s.w.end() || it->second.cols != HY_HIDDEN)
        return perr(HY_ERR_INVALID_ARGUMENT, what + ": no [ffn x 1024] layers.0.mlp.gate_proj");
    *ffn = it->second.rows;
    return HY_OK;
}

int open_pair(const std::string& root, const std::string& dir, const std::string& stem, Mapping* m, Slots* s)
{
    const std::string param = root + "/" + dir + "/" + stem + ".ncnn.param";
    const std::string bin = root + "/" + dir + "/" + stem + ".ncnn.bin";
    int rc = m->open(bin);
    if (rc) return rc;
    std::vector<std::pair<std::string, Weight>> named;
    if ((rc = read_weights(param, bin, *m, &named))) return rc;
    return collect(named, s);
}

int load_base(const std::string& root, Package* p)
{
    int rc;
    // The tied table: text_embed.ncnn.bin (the LM head's param points at the same bin).
    if ((rc = open_pair(root, "text_embed", "text_embed", &p->embed_bin, &p->embed))) return rc;
    auto e = p->embed.w.find(std::make_pair(-1, std::string("embed_tokens")));
    if (e == p->embed.w.end())
    {
        if (p->embed.w.size() != 1)
            return perr(HY_ERR_INVALID_ARGUMENT, "text_embed: expected one embedding table, found " +
                                                     std::to_string(p->embed.w.size()) + " named weights");
        e = p->embed.w.begin();
    }
    if (e->second.cols != HY_HIDDEN) return perr(HY_ERR_INVALID_ARGUMENT, "text_embed: the table is not [vocab x 1024]");
    p->vocab = e->second.rows;
    p->w.embed = e->second.a.data;
    if ((rc = open_pair(root, "text_decoder", "text_decoder_kv", &p->decoder_bin, &p->decoder))) return rc;
    p->layers = p->decoder.max_layer + 1;
    if (p->layers <= 0) return perr(HY_ERR_INVALID_ARGUMENT, "text_decoder: no decoder layers found");
    if ((rc = ffn_of(p->decoder, "text_decoder", &p->ffn))) return rc;
    p->lw.resize(p->layers);
    for (int l = 0; l < p->layers; ++l)
        if ((rc = layer_weights(p->decoder, l, p->ffn, "text_decoder", &p->lw[l]))) return rc;
    if ((rc = need(p->decoder, -1, "norm", HY_HIDDEN, 1, "text_decoder", &p->w.final_norm))) return rc;
    p->w.layers = p->lw.data();
    return HY_OK;
}

int load_draft(const std::string& root, int ffn, Package* p)
{
    int rc;
    if ((rc = open_pair(root, "dflash", "dflash", &p->draft_bin, &p->draft))) return rc;
    p->draft_layers = p->draft.max_layer + 1;
    if (p->draft_layers <= 0) return perr(HY_ERR_INVALID_ARGUMENT, "dflash: no draft layers found");
    p->dlw.resize(p->draft_layers);
    for (int l = 0; l < p->draft_layers; ++l)
        if ((rc = layer_weights(p->draft, l, ffn, "dflash", &p->dlw[l]))) return rc;
    if ((rc = need(p->draft, -1, "fc", HY_HIDDEN, HY_NUM_AUX_LAYERS * HY_HIDDEN, "dflash", &p->dw.fc))) return rc;
    if ((rc = need(p->draft, -1, "hidden_norm", HY_HIDDEN, 1, "dflash", &p->dw.hidden_norm))) return rc;
    if ((rc = need(p->draft, -1, "norm", HY_HIDDEN, 1, "dflash", &p->dw.norm))) return rc;
    p->dw.num_layers = p->draft_layers;
    p->dw.layers = p->dlw.data();
    return HY_OK;
}

const float* field_ptr(const hy_layer_weights& w, const std::string& f)
{
    if (f == "input_norm") return w.input_norm;
    if (f == "q_proj") return w.q_proj;
    if (f == "k_proj") return w.k_proj;
    if (f == "v_proj") return w.v_proj;
    if (f == "query_norm") return w.query_norm;
    if (f == "key_norm") return w.key_norm;
    if (f == "o_proj") return w.o_proj;
    if (f == "post_norm") return w.post_norm;
    if (f == "gate_proj") return w.gate_proj;
    if (f == "up_proj") return w.up_proj;
    if (f == "down_proj") return w.down_proj;
    return nullptr;
}

}  // namespace

extern "C" {

int hy_package_inspect(const char* model_root, int* num_layers, int* vocab_size, int* ffn_dim, int* draft_layers)
{
    if (!model_root) return perr(HY_ERR_INVALID_ARGUMENT, "null model root");
    Package p;
    int rc = load_base(model_root, &p);
    if (rc) return rc;
    int dl = 0;
    if (draft_layers)
    {
        struct stat st{};
        const std::string dparam = std::string(model_root) + "/dflash/dflash.ncnn.param";
        if (stat(dparam.c_str(), &st) == 0)
        {
            if ((rc = load_draft(model_root, p.ffn, &p))) return rc;
            dl = p.draft_layers;
        }
        *draft_layers = dl;
    }
    if (num_layers) *num_layers = p.layers;
    if (vocab_size) *vocab_size = p.vocab;
    if (ffn_dim) *ffn_dim = p.ffn;
    return HY_OK;
}

int hy_package_read_tensor(const char* model_root, int draft, int layer, const char* field, float* out, size_t capacity,
                           size_t* count)
{
    if (!model_root || !field) return perr(HY_ERR_INVALID_ARGUMENT, "null argument");
    Package p;
    int rc = load_base(model_root, &p);
    if (rc) return rc;
    if (draft && (rc = load_draft(model_root, p.ffn, &p))) return rc;
    const std::string f(field);
    const float* src = nullptr;
    size_t n = 0;
    auto lin = [&](int rows, int cols) { n = static_cast<size_t>(rows) * cols; };
    const int nl = draft ? p.draft_layers : p.layers;
    if (f == "embed") { src = p.w.embed; lin(p.vocab, HY_HIDDEN); }
    else if (f == "final_norm" && !draft) { src = p.w.final_norm; lin(HY_HIDDEN, 1); }
    else if (f == "norm" && draft) { src = p.dw.norm; lin(HY_HIDDEN, 1); }
    else if (f == "hidden_norm" && draft) { src = p.dw.hidden_norm; lin(HY_HIDDEN, 1); }
    else if (f == "fc" && draft) { src = p.dw.fc; lin(HY_HIDDEN, HY_NUM_AUX_LAYERS * HY_HIDDEN); }
    else
    {
        if (layer < 0 || layer >= nl) return perr(HY_ERR_INVALID_ARGUMENT, "layer out of range");
        src = field_ptr(draft ? p.dlw[layer] : p.lw[layer], f);
        if (!src) return perr(HY_ERR_INVALID_ARGUMENT, "unknown tensor " + f);
        const int q = HY_NUM_Q_HEADS * HY_HEAD_DIM, kv = HY_NUM_KV_HEADS * HY_HEAD_DIM;
        if (f == "q_proj") lin(q, HY_HIDDEN);
        else if (f == "k_proj" || f == "v_proj") lin(kv, HY_HIDDEN);
        else if (f == "o_proj") lin(HY_HIDDEN, q);
        else if (f == "gate_proj" || f == "up_proj") lin(p.ffn, HY_HIDDEN);
        else if (f == "down_proj") lin(HY_HIDDEN, p.ffn);
        else if (f == "query_norm" || f == "key_norm") lin(HY_HEAD_DIM, 1);
        else lin(HY_HIDDEN, 1);
    }
    if (count) *count = n;
    if (out)
    {
        if (capacity < n) return perr(HY_ERR_CAPACITY, "tensor " + f + " has " + std::to_string(n) + " values");
        std::memcpy(out, src, n * sizeof(float));
    }
    return HY_OK;
}

int hy_ctx_create_from_package(const hy_config* cfg, const char* model_root, hy_ctx** out)
{
    if (!cfg || !model_root || !out) return perr(HY_ERR_INVALID_ARGUMENT, "null argument");
    Package p;
    int rc = load_base(model_root, &p);
    if (rc) return rc;
    hy_config c = *cfg;
    c.num_layers = p.layers;
    c.vocab_size = p.vocab;
    c.ffn_dim = p.ffn;
    return hy_ctx_create(&c, &p.w, out);   // (its own message on failure)
}

int hy_draft_load_package(hy_ctx* ctx, const char* model_root, int mask_token)
{
    if (!ctx || !model_root) return perr(HY_ERR_INVALID_ARGUMENT, "null argument");
    hy_config cfg;
    int rc = hy_ctx_config(ctx, &cfg);
    if (rc) return rc;
    Package p;
    if ((rc = load_draft(model_root, cfg.ffn_dim, &p))) return rc;
    p.dw.mask_token = mask_token;
    return hy_draft_load(ctx, &p.dw);
}

}  // extern "C"
