"""Request-parallel batch decoding across GPUs (independent replicas).

The reference's JSONL batch driver (src/batch_jsonl.cpp `run_jsonl_batch`,
384-480; src/batch_jsonl.h:25-45) runs records sequentially through one
`HunyuanOCR`, calls a `BatchInfer` callback per record, writes one output
record per input record in input order (failures are records with
`ok: false`, stage and message) and returns a `BatchSummary` (total,
succeeded, failed).

Here the same contract is kept per process, and the records are partitioned
across GPUs: one process per GPU, each holding its own full copy of the
weights, takes the records with index i % world == rank. There is no
collective on the data path; the host gathers the per-rank results once at
the end (`gather_in_order`) and merges them in input order, which gives the
same output file as the sequential driver.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Iterable, List, Optional, Sequence


@dataclass
class BatchSummary:
    """src/batch_jsonl.h:27-31."""
    total: int = 0
    succeeded: int = 0
    failed: int = 0


@dataclass
class BatchRecord:
    """One output record: `ok` with the generated tokens, or the failing stage and message."""
    index: int
    id: str
    ok: bool
    tokens: List[int] = field(default_factory=list)
    stage: str = ""
    error: str = ""


def partition(n_records: int, world: int, rank: int) -> List[int]:
    """Record indices of one rank: round-robin by index (i mod world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    return list(range(rank, n_records, world))


def run_partition(records: Sequence, infer: Callable, world: int = 1, rank: int = 0,
                  record_id: Optional[Callable] = None,
                  channel: Optional["StoreChannel"] = None) -> tuple[List[BatchRecord], BatchSummary]:
    """Run this rank's records through `infer(record) -> tokens` (which raises on failure,
    like a BatchInfer returning false with a RuntimeError). Returns this rank's output
    records in input order and its summary. With a `channel`, every record is published
    as soon as it is done (and counts as this rank's heartbeat), and the rank reports
    that it finished after its last record."""
    out: List[BatchRecord] = []
    summary = BatchSummary()
    if channel is not None:
        channel.beat()
    for i in partition(len(records), world, rank):
        rid = record_id(records[i]) if record_id else str(i)
        summary.total += 1
        try:
            tokens = infer(records[i])
        except Exception as exc:  # noqa: BLE001 - every failure becomes an ok:false record
            summary.failed += 1
            stage = getattr(exc, "stage", "inference")
            out.append(BatchRecord(i, rid, False, stage=stage, error=str(exc) or "inference failed"))
        else:
            summary.succeeded += 1
            out.append(BatchRecord(i, rid, True, tokens=list(tokens)))
        if channel is not None:
            channel.publish(out[-1])
    if channel is not None:
        channel.finish()
    return out, summary


def run_partition_batched(records: Sequence, infer_many: Callable, world: int = 1, rank: int = 0,
                          record_id: Optional[Callable] = None) -> tuple[List[BatchRecord], BatchSummary]:
    """run_partition for a rank that decodes its records together (several sequences
    per GPU step): `infer_many(records) -> [(ok, tokens or error message)]`, one entry
    per record in order. Same output records and summary as run_partition."""
    idx = partition(len(records), world, rank)
    results = infer_many([records[i] for i in idx]) if idx else []
    if len(results) != len(idx):
        raise ValueError(f"infer_many returned {len(results)} results for {len(idx)} records")
    out: List[BatchRecord] = []
    summary = BatchSummary(total=len(idx))
    for i, (ok, value) in zip(idx, results):
        rid = record_id(records[i]) if record_id else str(i)
        if ok:
            summary.succeeded += 1
            out.append(BatchRecord(i, rid, True, tokens=list(value)))
        else:
            summary.failed += 1
            out.append(BatchRecord(i, rid, False, stage="inference", error=str(value) or "inference failed"))
    return out, summary


def merge_in_order(parts: Iterable[Sequence[BatchRecord]]) -> tuple[List[BatchRecord], BatchSummary]:
    """Merge per-rank outputs into input order and add up the summaries."""
    merged = sorted((r for p in parts for r in p), key=lambda r: r.index)
    for a, b in zip(merged, merged[1:]):
        if a.index == b.index:
            raise ValueError(f"record {a.index} was produced by two ranks")
    s = BatchSummary(total=len(merged), succeeded=sum(r.ok for r in merged),
                     failed=sum(not r.ok for r in merged))
    return merged, s


def gather_in_order(local: Sequence[BatchRecord], world: int, rank: int):
    """Gather every rank's records on rank 0 (torch.distributed object gather, once,
    after the work) and merge them in input order. Returns (records, summary) on
    rank 0 and (None, None) elsewhere."""
    if world == 1:
        return merge_in_order([local])
    import torch.distributed as dist

    parts = [None] * world if rank == 0 else None
    dist.gather_object(list(local), parts, dst=0)
    if rank != 0:
        return None, None
    return merge_in_order(parts)


class StoreChannel:
    """Per-record results and liveness of the ranks through the process group's
    key-value store, so that rank 0 can assemble the output without a collective
    that would wait forever for a rank that left.

    Every rank publishes each finished record (which also bumps its heartbeat
    counter) and a `done` flag after its last one. Rank 0 (`collect`) polls the
    store: a record appears when its rank published it; a rank whose heartbeat
    has not moved for `rank_timeout_s` seconds and that never reported `done`
    is taken to have left, and each of its unpublished records becomes an
    ok:false record (stage "rank") - the reference's per-record failure path,
    src/batch_jsonl.cpp:274-296, extended to a rank that is gone. The timeout
    must exceed the longest single infer call."""

    def __init__(self, store, world: int, rank: int, prefix: str = "hy_batch"):
        self.store, self.world, self.rank, self.prefix = store, world, rank, prefix

    @classmethod
    def from_default_group(cls, prefix: str = "hy_batch") -> "StoreChannel":
        import torch.distributed as dist
        return cls(dist.distributed_c10d._get_default_store(), dist.get_world_size(), dist.get_rank(), prefix)

    def _key(self, *parts) -> str:
        return "/".join((self.prefix,) + tuple(str(p) for p in parts))

    def beat(self) -> None:
        self.store.add(self._key("beat", self.rank), 1)

    def publish(self, rec: BatchRecord) -> None:
        import pickle
        self.store.set(self._key("rec", rec.index), pickle.dumps(rec))
        self.beat()

    def finish(self) -> None:
        self.store.set(self._key("done", self.rank), b"1")

    def collect(self, n_records: int, rank_timeout_s: float = 120.0, poll_s: float = 0.02,
                clock: Callable = None) -> tuple[List[BatchRecord], BatchSummary]:
        """On rank 0, after its own records: every record in input order and the summary.
        Returns once each record was published or its rank was found gone."""
        import pickle
        import time
        clock = clock or time.monotonic
        got = {}
        pending = set(range(n_records))
        last_beat = {r: None for r in range(self.world)}
        last_move = {r: clock() for r in range(self.world)}
        while pending:
            now = clock()
            for i in sorted(pending):
                k = self._key("rec", i)
                if self.store.check([k]):
                    got[i] = pickle.loads(self.store.get(k))
                    pending.discard(i)
            if not pending:
                break
            owners = {i % self.world for i in pending}
            for r in owners:
                beat = self.store.add(self._key("beat", r), 0)
                if beat != last_beat[r]:
                    last_beat[r], last_move[r] = beat, now
                done = self.store.check([self._key("done", r)])
                if done or now - last_move[r] > rank_timeout_s:
                    why = ("finished without publishing it" if done else
                           f"stopped responding (no progress for {rank_timeout_s:g} s)")
                    for i in [i for i in pending if i % self.world == r]:
                        k = self._key("rec", i)
                        if self.store.check([k]):   # published since the scan above
                            got[i] = pickle.loads(self.store.get(k))
                        else:
                            got[i] = BatchRecord(i, str(i), False, stage="rank", error=f"rank {r} {why}")
                        pending.discard(i)
            time.sleep(poll_s)
        return merge_in_order([[got[i] for i in range(n_records)]])
