"""Request partitioning across GPUs (CPU): round-robin assignment, per-record
failures, and the in-order merge on rank 0, with two gloo ranks as processes.

Mirrors the reference's batch contract (src/batch_jsonl.cpp:384-480: one output
record per input record, in input order; failed records are `ok: false`;
BatchSummary counts) and tests/batch_jsonl_test.cpp's use of an injected
inference callback.
"""
import importlib.util
import os
import socket
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _batch():
    if "hy_batch" in sys.modules:
        return sys.modules["hy_batch"]
    spec = importlib.util.spec_from_file_location("hy_batch", os.path.join(REPO, "hunyuanocr-ncnn_b200", "batch.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["hy_batch"] = mod   # dataclasses look their module up by name
    spec.loader.exec_module(mod)
    return mod


class _Fail(RuntimeError):
    stage = "decode"


def _infer(rec):
    # Injected callback: record 5 fails, the rest "decode" to a token list derived from the record.
    if rec == 5:
        raise _Fail("synthetic failure on record 5")
    return [rec, rec * 2 + 1]


def test_partition_round_robin_covers_every_record_once():
    b = _batch()
    for n in (0, 1, 7, 64):
        for world in (1, 2, 3, 8):
            parts = [b.partition(n, world, r) for r in range(world)]
            flat = sorted(i for p in parts for i in p)
            assert flat == list(range(n))
            for r, p in enumerate(parts):
                assert all(i % world == r for i in p)
    with pytest.raises(ValueError):
        b.partition(4, 2, 2)


def test_single_process_matches_sequential_contract():
    b = _batch()
    records = list(range(9))
    out, s = b.run_partition(records, _infer)
    merged, ms = b.merge_in_order([out])
    assert [r.index for r in merged] == records
    assert (ms.total, ms.succeeded, ms.failed) == (9, 8, 1)
    assert (s.total, s.succeeded, s.failed) == (9, 8, 1)
    bad = merged[5]
    assert not bad.ok and bad.stage == "decode" and "record 5" in bad.error
    assert merged[3].tokens == [3, 7]


def test_batched_partition_matches_per_record_contract():
    """Records decoded together (one infer_many call per rank) give the same output
    records and summaries as one record at a time."""
    b = _batch()
    records = list(range(11))

    def infer_many(recs):
        out = []
        for r in recs:
            try:
                out.append((True, _infer(r)))
            except _Fail as exc:
                out.append((False, str(exc)))
        return out

    for world in (1, 3):
        parts, seq_parts = [], []
        for rank in range(world):
            o1, s1 = b.run_partition_batched(records, infer_many, world=world, rank=rank)
            o2, s2 = b.run_partition(records, _infer, world=world, rank=rank)
            assert (s1.total, s1.succeeded, s1.failed) == (s2.total, s2.succeeded, s2.failed)
            parts.append(o1)
            seq_parts.append(o2)
        m1, t1 = b.merge_in_order(parts)
        m2, t2 = b.merge_in_order(seq_parts)
        assert [(r.index, r.ok, r.tokens) for r in m1] == [(r.index, r.ok, r.tokens) for r in m2]
        assert (t1.total, t1.succeeded, t1.failed) == (11, 10, 1)
    with pytest.raises(ValueError):
        b.run_partition_batched(records, lambda recs: [], world=1, rank=0)


def test_merge_rejects_duplicates():
    b = _batch()
    r = b.BatchRecord(1, "1", True, [1])
    with pytest.raises(ValueError):
        b.merge_in_order([[r], [r]])


def _worker(rank, world, port, n, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b = _batch()
        records = list(range(n))
        local, s = b.run_partition(records, _infer, world=world, rank=rank)
        merged, ms = b.gather_in_order(local, world, rank)
        if rank == 0:
            q.put(([(r.index, r.ok, r.tokens) for r in merged], (ms.total, ms.succeeded, ms.failed)))
        q.put(("rank", rank, [r.index for r in local], (s.total, s.succeeded, s.failed)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_merge_in_input_order():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n, world, port = 11, 2, _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    msgs = [q.get(timeout=60) for _ in range(world + 1)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ranks = {m[1]: m for m in msgs if m[0] == "rank"}
    assert ranks[0][2] == list(range(0, n, 2)) and ranks[1][2] == list(range(1, n, 2))
    merged, summary = next(m for m in msgs if m[0] != "rank")
    assert [i for i, _, _ in merged] == list(range(n))
    assert summary == (n, n - 1, 1)
    assert all(ok == (i != 5) for i, ok, _ in merged)
    assert merged[4][2] == [4, 9]


def _leaving_worker(rank, world, port, n, q):
    """Rank 1 finishes one record, then leaves without a word (between records);
    rank 0 must still return every record: rank 1's first as published, the rest
    as ok:false rank failures, within the rank timeout."""
    import datetime
    import time
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    b = _batch()
    ch = b.StoreChannel.from_default_group(prefix="leave")
    records = list(range(n))
    if rank == 1:
        calls = []

        def infer(i):
            if calls:
                q.put(("left", rank))
                q.close()
                q.join_thread()   # the message is out before the process ends
                os._exit(0)    # the rank is gone: no more records, no done flag, no goodbye
            calls.append(i)
            return _infer(i)

        b.run_partition(records, infer, world=world, rank=rank, channel=ch)
        return
    t0 = time.monotonic()
    local, _ = b.run_partition(records, _infer, world=world, rank=rank, channel=ch)
    merged, summary = ch.collect(n, rank_timeout_s=3.0)
    q.put(("merged", [(r.index, r.ok, r.stage, r.tokens) for r in merged],
           (summary.total, summary.succeeded, summary.failed), time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)   # the peer is gone: skip the process-group teardown


def test_rank_leaving_between_records_gives_failure_records():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n, world, port = 9, 2, _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    msgs = [q.get(timeout=90) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert ("left", 1) in msgs
    _, merged, summary, seconds = next(m for m in msgs if m[0] == "merged")
    assert [i for i, *_ in merged] == list(range(n))
    # Rank 0 (even records): its own results. Rank 1 (odd records): record 1
    # published before it left; 3, 5, 7 rank failures.
    for i, ok, stage, toks in merged:
        if i % 2 == 0:
            assert ok and toks == _infer(i)
        elif i == 1:
            assert ok and toks == _infer(1)
        else:
            assert not ok and stage == "rank", (i, ok, stage)
    assert summary == (n, 5 + 1, 3)
    assert seconds < 30
