"""Host logic of the vocab-sharded sampler on CPU ranks (gloo, world size 2 and 3).

The device steps are replaced by a stand-in that writes rank-tagged records, checks that the
all-gather delivered them in rank order, answers resolved rows from the CPU oracle on the full
row, and flags chosen rows as unresolved. The tests check that every rank returns the same ids,
that they equal the oracle's, and that the fallback rebuilt each unresolved row -- logits,
parameters, uniform and history -- exactly from the shards.

Failure handling, made on the host: a rank that exits between steps (the survivors' next step
must raise within the process group's timeout), and a rank that raises inside the fallback
(every rank must raise, none may hang).
"""

from __future__ import annotations

import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import oracle_row
from vinfer_b200.sampling import RowParams, TokenHistogram
from vinfer_b200.sharded import ShardedSampler, select_rows, shard_range
from vinfer_b200.workloads import Workload, make


class FakeShardKernels:
    def __init__(self, w: Workload, unresolved_rows: set[int]) -> None:
        self.w = w
        self.unresolved_rows = unresolved_rows
        self.full_calls: list[dict] = []

    def record_bytes(self, cap: int) -> int:
        return 32 + 8 * cap

    def local(self, logits, params, uniforms, history, voff, vtotal, cap, records, scratch):
        rank = dist.get_rank()
        records.fill_(rank + 1)
        records[:8] = torch.tensor([voff], dtype=torch.int64).view(torch.uint8)

    def merge(self, logits, params, uniforms, history, voff, vtotal, cap, gathered, world, out,
              unresolved, probs_out):
        n = gathered.numel() // world
        for r in range(world):
            part = gathered[r * n:(r + 1) * n]
            assert int(part[:8].view(torch.int64)) == shard_range(vtotal, world, r)[0]
            assert bool((part[8:] == r + 1).all())
        for row in range(self.w.batch):
            if row in self.unresolved_rows:
                unresolved[row] = 1
                out[row] = -1
            else:
                unresolved[row] = 0
                out[row] = oracle_row(self.w, row).token

    def full(self, logits, params, uniforms, history, out, probs_out):
        self.full_calls.append({"logits": logits.clone(), "params": params, "u": uniforms,
                                "hist": history})
        sub = Workload("sub", logits.clone(), params.temperature.numpy(), params.top_k.numpy(),
                       params.top_p.numpy(), params.min_p.numpy(),
                       params.repetition_penalty.numpy(), params.presence_penalty.numpy(),
                       params.frequency_penalty.numpy(), uniforms.numpy())
        if history is not None:
            sub.hist_row_ptr = history.row_ptr.numpy()
            sub.hist_ids = history.ids.numpy()
            sub.hist_counts = history.counts.numpy()
        for i in range(sub.batch):
            out[i] = oracle_row(sub, i).token

    def check(self) -> None:
        pass


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, config: int, batch: int, vocab: int,
               unresolved: list[int], results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = make(config, batch=batch, vocab=vocab)
        lo, hi = shard_range(vocab, world, rank)
        shard = w.logits[:, lo:hi].contiguous()
        params = RowParams.from_arrays("cpu", **w.param_arrays())
        u = torch.from_numpy(w.uniforms)
        hist = None
        if w.hist_row_ptr is not None:
            hist = TokenHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, "cpu")
        k = FakeShardKernels(w, set(unresolved))
        s = ShardedSampler(k, record_cap=8)
        ids = s.sample_batch(shard, params, u, hist, vocab)
        want = np.array([oracle_row(w, r).token for r in range(w.batch)])
        assert np.array_equal(ids.numpy(), want), (ids.numpy(), want)
        assert s.last_unresolved == len(unresolved)
        if unresolved:
            call = k.full_calls[0]
            idx = torch.tensor(sorted(unresolved))
            assert torch.equal(call["logits"], w.logits.index_select(0, idx))
            assert torch.equal(call["u"], u.index_select(0, idx))
            for name in ("temperature", "top_k", "top_p", "repetition_penalty"):
                assert torch.equal(getattr(call["params"], name),
                                   getattr(params, name).index_select(0, idx))
            if hist is not None:
                for j, r in enumerate(sorted(unresolved)):
                    a, b = int(w.hist_row_ptr[r]), int(w.hist_row_ptr[r + 1])
                    h = call["hist"]
                    c, d = int(h.row_ptr[j]), int(h.row_ptr[j + 1])
                    assert np.array_equal(h.ids[c:d].numpy(), w.hist_ids[a:b])
                    assert np.array_equal(h.counts[c:d].numpy(), w.hist_counts[a:b])
        else:
            assert not k.full_calls
        gathered = [None] * world
        dist.all_gather_object(gathered, ids.tolist())
        assert all(g == gathered[0] for g in gathered)
        # the device steps alone: no fallback, unresolved rows left at -1 and counted
        s.pending_unresolved(shard.device)
        for _ in range(2):
            ids2 = s.sample_batch_async(shard, params, u, hist, vocab)
        assert s.pending_unresolved(shard.device) == 2 * len(unresolved)
        assert s.pending_unresolved(shard.device) == 0
        keep = [r for r in range(w.batch) if r not in unresolved]
        assert np.array_equal(ids2.numpy()[keep], want[keep])
        assert all(int(ids2[r]) == -1 for r in unresolved)
        results.put((rank, "ok"))
    except Exception as exc:  # reported to the parent, which fails the test
        results.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,config,unresolved", [
    (2, 3, [1, 4]),   # penalties with histories; two rows take the fallback
    (2, 2, []),       # heterogeneous rows, all resolved from the records
    (3, 3, [0, 5]),   # uneven shards (1000 over 3 ranks)
])
def test_sharded_host_logic_on_gloo_ranks(world, config, unresolved):
    ctx = mp.get_context("spawn")
    results = ctx.SimpleQueue()
    mp.start_processes(_rank_main, args=(world, _free_port(), config, 6, 1000, unresolved,
                                         results), nprocs=world, join=True,
                       start_method="spawn")
    got = sorted(results.get() for _ in range(world))
    assert got == [(r, "ok") for r in range(world)], got


class FailingFullKernels(FakeShardKernels):
    """Stand-in whose unsharded fallback raises on one rank (after the rows' all-gather)."""

    def __init__(self, w: Workload, unresolved_rows: set[int], failing_rank: int) -> None:
        super().__init__(w, unresolved_rows)
        self.failing_rank = failing_rank

    def full(self, logits, params, uniforms, history, out, probs_out):
        if dist.get_rank() == self.failing_rank:
            raise RuntimeError("injected failure in the fallback")
        super().full(logits, params, uniforms, history, out, probs_out)


PG_TIMEOUT_S = 6


def _failure_rank_main(rank: int, world: int, port: int, scenario: str, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    w = make(3, batch=4, vocab=600)
    lo, hi = shard_range(600, world, rank)
    shard = w.logits[:, lo:hi].contiguous()
    params = RowParams.from_arrays("cpu", **w.param_arrays())
    u = torch.from_numpy(w.uniforms)
    hist = TokenHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, "cpu")
    if scenario == "leave":
        s = ShardedSampler(FakeShardKernels(w, set()), record_cap=8)
        s.sample_batch(shard, params, u, hist, 600)  # one full step on every rank
        if rank == world - 1:
            results.put((rank, "left"))
            os._exit(0)  # leaves between steps: no collective of its own is in flight
        t0 = time.monotonic()
        try:
            s.sample_batch(shard, params, u, hist, 600)
            results.put((rank, "no error"))
        except Exception as exc:  # noqa: BLE001 -- the expected outcome
            results.put((rank, f"raised after {time.monotonic() - t0:.1f}s: "
                               f"{type(exc).__name__}"))
        os._exit(0)  # the group lost a member: skip its teardown
    else:  # "fallback": rank 1 raises inside the unsharded fallback
        s = ShardedSampler(FailingFullKernels(w, {1, 2}, failing_rank=1), record_cap=8)
        try:
            s.sample_batch(shard, params, u, hist, 600)
            results.put((rank, "no error"))
        except Exception as exc:  # noqa: BLE001 -- the expected outcome
            results.put((rank, f"raised: {exc}"))
        dist.destroy_process_group()


def _run_failure(world: int, scenario: str) -> list[tuple[int, str]]:
    ctx = mp.get_context("spawn")
    results = ctx.SimpleQueue()
    t0 = time.monotonic()
    mp.start_processes(_failure_rank_main, args=(world, _free_port(), scenario, results),
                       nprocs=world, join=True, start_method="spawn")
    out = sorted(results.get() for _ in range(world))
    # every rank ended well within a few process-group timeouts: nobody hung
    assert time.monotonic() - t0 < 60 + 3 * PG_TIMEOUT_S
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_a_rank_that_leaves_between_steps_fails_the_survivors_next_step(world):
    got = _run_failure(world, "leave")
    assert got[-1] == (world - 1, "left")
    for rank, msg in got[:-1]:
        assert msg.startswith("raised after"), (rank, msg)
        # an error within the process group's timeout (plus scheduling slack), not a hang
        assert float(msg.split()[2].rstrip("s:")) <= PG_TIMEOUT_S + 10, msg


def test_a_rank_that_raises_in_the_fallback_fails_every_rank():
    got = _run_failure(2, "fallback")
    assert got[0][0] == 0 and "rank(s) failed while resolving rows [1, 2]" in got[0][1], got
    assert got[1][0] == 1 and "injected failure in the fallback" in got[1][1], got


def test_select_rows_rebuilds_histories():
    w = make(3, batch=5, vocab=500)
    params = RowParams.from_arrays("cpu", **w.param_arrays())
    hist = TokenHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, "cpu")
    idx = torch.tensor([4, 0, 2])
    p, u, h = select_rows(params, torch.from_numpy(w.uniforms), hist, idx)
    assert torch.equal(p.top_k, params.top_k[idx])
    assert torch.equal(u, torch.from_numpy(w.uniforms)[idx])
    for j, r in enumerate([4, 0, 2]):
        a, b = int(w.hist_row_ptr[r]), int(w.hist_row_ptr[r + 1])
        c, d = int(h.row_ptr[j]), int(h.row_ptr[j + 1])
        assert np.array_equal(h.ids[c:d].numpy(), w.hist_ids[a:b])


def test_shard_ranges_cover_the_vocabulary():
    for V in (7, 1000, 248_320):
        for world in (1, 2, 3, 8):
            spans = [shard_range(V, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == V
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
    with pytest.raises(ValueError):
        shard_range(100, 2, 2)
