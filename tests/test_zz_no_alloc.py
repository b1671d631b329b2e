"""hy_lm_head_select_noalloc: the LM-head select on device buffers, for callers
that cannot allocate device memory while they decode (their memory is held by
their own caching allocator, or a cudaMalloc/cudaFree would synchronise a GPU
shared with other streams). Its argmax scratch is a static device-global array.

It has no reference counterpart; its reference is the library's own
hy_lm_head_select (run_lm_head + select_logit_rows, src/text_runtime.cpp:430-439,
757-797), whose argmax indices the parity tests require bit-exact. The file is
named to be collected last, and it passes alone in a fresh process too.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PENALTY = 1.08


def _runtime(pkg):
    # Full vocabulary (the real launch shape), two layers (the decoder is not used here).
    return pkg.TextRuntime.synthetic(seed=11, num_layers=2, max_prefill=64, max_tokens=32, max_context=256)


def test_noalloc_select_matches_existing_entry_point(pkg):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(2024)
    with _runtime(pkg) as rt:
        # Penalty history that the selection must honour (ids that score high on
        # some rows get divided / multiplied by the penalty).
        rt.set_history([int(t) for t in rng.integers(0, rt.cfg.vocab_size, size=64)])
        for rows in (1, 5, 16):
            hidden = rng.standard_normal((rows, 1024)).astype(np.float32)
            ref_tok, ref_raw, _ = rt.select_logit_rows(hidden, PENALTY)
            d_hidden = torch.from_numpy(hidden).to("cuda")
            d_tok = torch.empty(rows, dtype=torch.int32, device="cuda")
            d_raw = torch.empty(rows, dtype=torch.int32, device="cuda")
            for _ in range(2):   # two calls in a row: the scratch is reused
                d_tok.fill_(-1)
                d_raw.fill_(-1)
                torch.cuda.synchronize()
                free_before = torch.cuda.mem_get_info()[0]
                rt.select_logit_rows_noalloc(d_hidden.data_ptr(), rows, PENALTY, d_tok.data_ptr(), d_raw.data_ptr())
                # The call has returned only after the select finished: the
                # outputs are read without another synchronisation.
                np.testing.assert_array_equal(d_tok.cpu().numpy(), ref_tok)
                np.testing.assert_array_equal(d_raw.cpu().numpy(), ref_raw)
                # Nothing was allocated on the device (free memory did not drop).
                assert torch.cuda.mem_get_info()[0] >= free_before


def test_noalloc_select_ordered_by_event(pkg):
    """hidden_dev written by the caller's own stream and fenced with an event
    that the context's stream waits on (no host synchronisation before the call)."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(77)
    with _runtime(pkg) as rt:
        rt.set_history([int(t) for t in rng.integers(0, rt.cfg.vocab_size, size=32)])
        ctx_stream = torch.cuda.ExternalStream(rt.stream)
        producer = torch.cuda.Stream()
        for rows in (1, 16):
            hidden = rng.standard_normal((rows, 1024)).astype(np.float32)
            ref_tok, ref_raw, _ = rt.select_logit_rows(hidden, PENALTY)
            src = torch.from_numpy(hidden).pin_memory()
            d_hidden = torch.empty((rows, 1024), dtype=torch.float32, device="cuda")
            d_tok = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
            d_raw = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            with torch.cuda.stream(producer):
                d_hidden.zero_()
                d_hidden.copy_(src, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(producer)
            ctx_stream.wait_event(ready)
            rt.select_logit_rows_noalloc(d_hidden.data_ptr(), rows, PENALTY, d_tok.data_ptr(), d_raw.data_ptr())
            np.testing.assert_array_equal(d_tok.cpu().numpy(), ref_tok)
            np.testing.assert_array_equal(d_raw.cpu().numpy(), ref_raw)


def test_noalloc_select_rejects_sizes_beyond_scratch(pkg):
    torch = pytest.importorskip("torch")
    with _runtime(pkg) as rt:
        d_hidden = torch.zeros((17, 1024), dtype=torch.float32, device="cuda")
        d_out = torch.zeros(17, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        with pytest.raises(pkg.HyError, match="rows must be in 1..16"):
            rt.select_logit_rows_noalloc(d_hidden.data_ptr(), 17, PENALTY, d_out.data_ptr(), d_out.data_ptr())
