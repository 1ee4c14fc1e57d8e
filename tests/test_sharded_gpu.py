"""Vocab-sharded sampling kernels against the CPU oracle, all ranks emulated on one GPU.

Each rank's ``vinfer_sample_local`` runs on its column slice of the full logits, the records are
laid out in rank order exactly as the all-gather delivers them, and ``vinfer_sample_merge`` runs
once per rank (each with its own shard for the probability slice). Every rank must produce the
same ids; rows flagged unresolved are finished with ``vinfer_sample`` on the full row, as the
sharded sampler does. The assembled ids and probabilities are compared with the oracle under
the same rules as the unsharded kernel.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import compare, report, to_device
from vinfer_b200 import SAMPLER, BackendContext
from vinfer_b200.sharded import B200ShardKernels, select_rows, shard_range
from vinfer_b200.workloads import make

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def backend():
    return SAMPLER.resolve("b200", BackendContext(torch.device("cuda", 0), torch.bfloat16))


def emulate(backend, w, world: int, cap: int = 64):
    dev = backend.device
    kern = B200ShardKernels(backend)
    lg, params, u, hist = to_device(w, dev)
    B, V = w.batch, w.vocab
    rec = kern.record_bytes(cap)
    gathered = torch.empty(world * B * rec, dtype=torch.uint8, device=dev)
    scratch = torch.empty(B, dtype=torch.int32, device=dev)
    for r in range(world):
        lo, hi = shard_range(V, world, r)
        kern.local(lg[:, lo:hi], params, u, hist, lo, V, cap,
                   gathered[r * B * rec:(r + 1) * B * rec], scratch)
    ids_per_rank, probs, unresolved = [], torch.empty(B, V, dtype=torch.float32, device=dev), None
    for r in range(world):
        lo, hi = shard_range(V, world, r)
        out = torch.full((B,), -7, dtype=torch.int32, device=dev)
        unres = torch.full((B,), -7, dtype=torch.int32, device=dev)
        pslice = torch.empty(B, hi - lo, dtype=torch.float32, device=dev)
        kern.merge(lg[:, lo:hi], params, u, hist, lo, V, cap, gathered, world, out, unres, pslice)
        probs[:, lo:hi] = pslice
        ids_per_rank.append(out.cpu().numpy())
        if unresolved is None:
            unresolved = unres.cpu().numpy()
        else:
            assert np.array_equal(unresolved, unres.cpu().numpy())
    torch.cuda.synchronize()
    backend.check()
    for r in range(1, world):
        assert np.array_equal(ids_per_rank[0], ids_per_rank[r])
    ids = ids_per_rank[0].copy()
    idx_np = np.nonzero(unresolved)[0]
    if idx_np.size:
        idx = torch.from_numpy(idx_np).to(dev)
        sp, su, sh = select_rows(params, u, hist, idx)
        fo = torch.empty(idx_np.size, dtype=torch.int32, device=dev)
        fp = torch.empty(idx_np.size, V, dtype=torch.float32, device=dev)
        backend.sample_batch(lg.index_select(0, idx).contiguous(), sp, su, sh, out=fo,
                             probs_out=fp)
        ids[idx_np] = fo.cpu().numpy()
        probs[idx] = fp
    torch.cuda.synchronize()
    backend.check()
    return ids, probs.cpu().numpy(), int(idx_np.size)


@pytest.mark.parametrize("config,batch,world", [
    (4, 32, 2), (4, 32, 8),      # the sharded benchmark configuration
    (3, 16, 4),                  # penalties: each rank applies the history entries of its shard
    (2, 32, 8),                  # greedy / top-k off / min-p rows
    (5, 16, 2),                  # top-k up to 1000: records overflow, rows take the fallback
    (1, 1, 3),                   # float32, uneven shards
])
def test_sharded_kernels_match_the_oracle(backend, config, batch, world):
    w = make(config, batch=batch)
    ids, probs, n_unres = emulate(backend, w, world)
    rep = compare(w, ids, probs)
    report(f"config {config} over {world} shards (batch {batch}), {n_unres} rows via the "
           "full-row path", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])


def test_config4_rows_resolve_from_the_records(backend):
    # top-k 50 bounds the kept set by the gathered candidates: no fallback
    w = make(4, batch=64)
    ids, probs, n_unres = emulate(backend, w, 4)
    assert n_unres == 0
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])
