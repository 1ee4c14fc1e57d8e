"""B200 sampler parity against the CPU oracle, through the C ABI (GPU only).

Seeded inputs of the five benchmark configurations at reduced batch but full vocabulary, small
hand-made vocabularies that reach every branch (ragged tails, ties, -inf, strided and
misaligned rows, penalties, min-p), the exact multi-pass search checked against the fast
path, and size-independent properties at the full config-3 batch.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import ctypes as C

from tests.helpers import compare, oracle_row, report, run_b200, to_device
from vinfer_b200 import SAMPLER, BackendContext, SamplingParams, position_uniform
from vinfer_b200 import _lib
from vinfer_b200.sampling import RowParams
from vinfer_b200.workloads import Workload, make

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def backend():
    return SAMPLER.resolve("b200", BackendContext(torch.device("cuda", 0), torch.bfloat16))


def _workload(x: torch.Tensor, params: list[dict], seed: int = 0, hist=None) -> Workload:
    B = x.shape[0]
    g = np.random.default_rng(seed)

    def col(name, default, dt=np.float32):
        return np.array([p.get(name, default) for p in params], dtype=dt)

    w = Workload("custom", x, col("temperature", 1.0), col("top_k", 0, np.int32),
                 col("top_p", 1.0), col("min_p", 0.0), col("repetition_penalty", 1.0),
                 col("presence_penalty", 0.0), col("frequency_penalty", 0.0),
                 g.random(B).astype(np.float32))
    if hist is not None:
        w.hist_row_ptr, w.hist_ids, w.hist_counts = hist
    return w


GRID = [
    {"temperature": 0.0},
    {"temperature": 1.0},
    {"temperature": 0.7, "top_k": 1},
    {"temperature": 0.7, "top_k": 3},
    {"temperature": 1.3, "top_k": 20},
    {"temperature": 0.5, "top_p": 0.8},
    {"temperature": 1.0, "top_p": 0.3},
    {"temperature": 0.9, "top_k": 50, "top_p": 0.9},
    {"temperature": 1.0, "min_p": 0.05},
    {"temperature": 0.6, "top_k": 20, "top_p": 0.95, "min_p": 0.1},
    {"temperature": 2.0, "top_p": 0.999},
    {"temperature": 0.2, "top_k": 300},
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=str)
@pytest.mark.parametrize("V", [6, 7, 96, 1000, 4097, 40000])
def test_small_vocabularies_match_the_oracle(backend, V, dtype):
    g = torch.Generator().manual_seed(V)
    B = len(GRID)
    x = (torch.randn(B, V, generator=g) * 2.0).to(dtype)
    w = _workload(x, GRID, seed=V)
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=str)
def test_penalties_match_the_oracle(backend, dtype):
    V = 5000
    g = torch.Generator().manual_seed(7)
    params = [dict(p, repetition_penalty=1.3, presence_penalty=0.4, frequency_penalty=0.2)
              for p in GRID]
    B = len(params)
    x = (torch.randn(B, V, generator=g) * 2.0).to(dtype)
    rng = np.random.default_rng(1)
    rows = []
    for r in range(B):
        # the top logits are the most likely to be penalised, so the penalties change ranks
        top = torch.topk(x[r].float(), 40).indices.numpy()
        rows.append(np.concatenate([top[::2], rng.integers(0, V, 200)]))
    ptr, ids_, cnt = [0], [], []
    for t in rows:
        u, c = np.unique(t, return_counts=True)
        ids_.append(u.astype(np.int32))
        cnt.append(c.astype(np.int32))
        ptr.append(ptr[-1] + len(u))
    w = _workload(x, params, hist=(np.array(ptr), np.concatenate(ids_), np.concatenate(cnt)))
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])


@pytest.mark.parametrize("config,batch", [(1, None), (2, 24), (3, 16), (5, 16)])
def test_benchmark_configs_match_the_oracle(backend, config, batch):
    w = make(config, batch=batch)
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    report(f"config {config} (batch {w.batch})", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])


def test_config5_every_row_class(backend):
    w = make(5, batch=32)  # eight rows of each class: flat, dominant, 1000-way tie, normal
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    report("config 5 row classes (batch 32)", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])


@pytest.mark.parametrize("config,batch", [(2, 24), (3, 16)])
def test_exact_search_agrees_with_the_fast_path(backend, config, batch):
    w = make(config, batch=batch)
    ids_fast, p_fast = run_b200(backend, w)
    ids_exact, p_exact = run_b200(backend, w, exact=True)
    same = ids_fast == ids_exact
    for r in np.nonzero(~same)[0]:
        assert oracle_row(w, int(r)).boundary, f"row {r}: fast {ids_fast[r]} exact {ids_exact[r]}"
    np.testing.assert_allclose(p_exact, p_fast, rtol=2e-5, atol=1e-30)


def test_ties_flat_rows_and_masked_logits(backend):
    V = 3000
    x = torch.randn(8, V, generator=torch.Generator().manual_seed(3))
    x[0] = 0.5  # flat
    x[1, :] = -1.0
    x[1, 100:400] = 2.0  # 300-way tie at the max
    x[2, 1::2] = float("-inf")  # masked half of the vocabulary
    x[3, :] = -0.0
    x[3, ::3] = 0.0  # signed zeros compare equal
    x[4, 10] = 40.0  # one dominant token
    x[5, 2500:] = float("-inf")
    x[6, ::7] = 3.0
    params = [{"temperature": 1.0, "top_p": 0.37}, {"temperature": 0.8, "top_k": 5},
              {"temperature": 1.0, "top_k": 10}, {"temperature": 1.0, "top_p": 0.5},
              {"temperature": 0.5, "top_p": 0.9}, {"temperature": 1.0, "top_k": 2999},
              {"temperature": 1.0, "top_k": 100, "top_p": 0.6}, {"temperature": 0.0}]
    for dtype in (torch.float32, torch.bfloat16):
        w = _workload(x.to(dtype), params, seed=5)
        for exact in (False, True):
            ids, probs = run_b200(backend, w, exact=exact)
            rep = compare(w, ids, probs)
            assert not rep.failures, (dtype, exact, str(rep), rep.failures[:5])


def test_strided_and_misaligned_rows(backend):
    w = make(2, batch=8, vocab=20001)
    ids_ref, _ = run_b200(backend, w, probs=False)
    for dtype in (torch.bfloat16, torch.float32):
        w2 = make(2, batch=8, vocab=20001)
        w2.logits = w2.logits.to(dtype)
        ids_c, _ = run_b200(backend, w2, probs=False)
        if dtype == torch.bfloat16:
            np.testing.assert_array_equal(ids_c, ids_ref)
        # rows with a larger stride, starting 1..3 elements past an aligned address
        for shift in (1, 3):
            big = torch.full((8, 20001 + 37), float("nan"), dtype=dtype, device=backend.device)
            big[:, shift:shift + 20001] = w2.logits.to(backend.device)
            view = big[:, shift:shift + 20001]
            ids_v, _ = run_b200(backend, w2, probs=False, logits=view)
            np.testing.assert_array_equal(ids_v, ids_c)


def test_full_batch_config3_is_deterministic_and_valid(backend):
    w = make(3)
    lg, params, u, hist = to_device(w, backend.device)
    a = backend.sample_batch(lg, params, u, hist).cpu().numpy()
    b = backend.sample_batch(lg, params, u, hist).cpu().numpy()
    backend.check()
    np.testing.assert_array_equal(a, b)
    assert ((a >= 0) & (a < w.vocab)).all()
    rep = compare(w, a, None)  # every one of the 256 rows
    report("config 3 ids, repeated call (batch 256)", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])


@pytest.mark.parametrize("config", [2, 3, 5])
def test_full_batch_configs_match_the_oracle(backend, config):
    # the benchmark configurations at their full batch (64 / 256 / 512 rows): every row's id
    # and every row's final probabilities against the oracle
    w = make(config)
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    report(f"config {config} full batch ({w.batch} rows)", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])


def test_config4_unsharded_at_full_vocabulary(backend):
    # configuration 4's rows (vocab 248,320, top-k 50, top-p 0.9) through vinfer_sample on one
    # GPU: the single-GPU reference the sharded runs are compared with
    w = make(4, batch=128)
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    report("config 4 unsharded (batch 128, vocab 248320)", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])


def test_one_workspace_serves_calls_of_different_shapes(backend):
    # A workspace sized for the larger shape, used by 8 rows and then 24 rows (and 8 again):
    # the per-row arrival counters sit in a header whose place does not depend on the shape,
    # so no call finds another's records over its counters.
    lib = backend.lib
    small, large = make(3, batch=8), make(3, batch=24, seed=9)
    nbytes = lib.vinfer_sampler_workspace_bytes(24, small.vocab, _lib.DTYPE_BF16)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=backend.device)
    _lib.check(lib.vinfer_sampler_workspace_init(ws.data_ptr(), nbytes, backend._stream()),
               "workspace init")
    for w in (small, large, small, large):
        lg, params, u, hist = to_device(w, backend.device)
        out = torch.full((w.batch,), -7, dtype=torch.int32, device=backend.device)
        a = backend.args(lg, params, u, hist, out, None)
        _lib.check(lib.vinfer_sample(C.byref(a), ws.data_ptr(), nbytes, backend._stream()),
                   "vinfer_sample")
        torch.cuda.synchronize()
        backend.check()
        rep = compare(w, out.cpu().numpy(), None)
        assert not rep.failures, (w.batch, str(rep), rep.failures[:5])


def test_single_row_api_uses_the_position_uniform(backend):
    w = make(1)
    x = w.logits[0].to(backend.device)
    p = SamplingParams(temperature=0.7, top_k=20, top_p=0.8)
    for pos in range(20):
        tok = backend.sample(x, p, seed=11, position=pos)
        w.uniforms[0] = np.float32(position_uniform(11, pos))
        w.hist_row_ptr = None
        w.repetition_penalty[0] = 1.0
        res = oracle_row(w, 0)
        assert res.boundary or tok == res.token


def test_invalid_row_parameters_are_reported(backend):
    V = 100
    x = torch.randn(3, V, device=backend.device)
    params = RowParams.from_arrays(backend.device, temperature=np.array([1.0, 1.0, -1.0]),
                                   top_p=np.array([1.0, 0.0, 1.0]))
    u = torch.full((3,), 0.5, device=backend.device)
    ids = backend.sample_batch(x, params, u).cpu().numpy()
    assert ids[0] >= 0 and ids[1] == -1 and ids[2] == -1
    with pytest.raises(RuntimeError, match="invalid sampling parameters"):
        backend.check()


def test_host_side_argument_errors_do_not_launch(backend):
    x = torch.randn(2, 10, device=backend.device)
    params = RowParams.from_arrays(backend.device, temperature=np.array([1.0]))
    with pytest.raises(ValueError):
        backend.sample_batch(x, params, torch.zeros(2, device=backend.device))
    assert _lib.load().vinfer_sample(None, None, 0, None) == _lib.E_ARG


def _hist_csr(rows):
    ptr, ids_, cnt = [0], [], []
    for t in rows:
        u, c = np.unique(np.asarray(t, np.int64), return_counts=True)
        ids_.append(u.astype(np.int32))
        cnt.append(c.astype(np.int32))
        ptr.append(ptr[-1] + len(u))
    return np.array(ptr, np.int64), np.concatenate(ids_), np.concatenate(cnt)


@pytest.mark.parametrize("batch", [600, 601])
def test_large_batch_rows_split_across_ctas(backend, batch):
    # more rows than resident CTAs: each CTA takes ceil(B / CTAs) rows' worth of the row-major
    # segment list. 600 rows are whole rows per CTA; with 601 the CTAs' ranges cut rows, whose
    # runs are finished by the CTA completing the row (records merged from two CTAs)
    w = make(2, batch=batch, vocab=20_000)
    ids, probs = run_b200(backend, w, probs=False)
    rows = list(range(0, batch, 7)) + [batch - 1]
    rep = compare(w, ids, None, rows=rows)
    assert not rep.failures, (str(rep), rep.failures[:5])


def test_long_histories_beyond_the_staging_areas(backend):
    # 3,000 and 5,000 distinct history ids: beyond the finishing kernel's staging (exact
    # search) and, for the second, beyond the streaming kernel's (global-memory lookups)
    V = 40_000
    g = torch.Generator().manual_seed(11)
    params = [dict(temperature=0.8, top_k=20, top_p=0.9, repetition_penalty=1.2,
                   presence_penalty=0.3, frequency_penalty=0.1),
              dict(temperature=1.0, top_k=0, top_p=0.8, repetition_penalty=0.9,
                   presence_penalty=-0.2, frequency_penalty=0.05),
              dict(temperature=0.0, repetition_penalty=1.5)]
    x = (torch.randn(len(params), V, generator=g) * 2.0).to(torch.bfloat16)
    rng = np.random.default_rng(2)
    rows = [rng.choice(V, 3000, replace=False), rng.choice(V, 5000, replace=False),
            rng.choice(V, 4500, replace=False)]
    w = _workload(x, params, hist=_hist_csr(rows))
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])


def test_small_batch_split_many_ways_with_penalties(backend):
    # four rows over the whole device: each row is cut into dozens of runs
    w = make(3, batch=4)
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])


@pytest.mark.parametrize("k", [32, 33, 64, 192, 193])
def test_top_k_around_the_candidate_path_limits(backend, k):
    V = 30_000
    g = torch.Generator().manual_seed(k)
    params = [dict(temperature=0.9, top_k=k), dict(temperature=1.2, top_k=k, top_p=0.7),
              dict(temperature=0.5, top_k=k, min_p=0.02)]
    x = (torch.randn(len(params), V, generator=g) * 1.5).float()
    w = _workload(x, params, seed=k)
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])


def test_penalised_rows_without_top_k(backend):
    # the online softmax sum corrected for penalised tokens (raw terms out, exact terms in)
    V = 50_000
    g = torch.Generator().manual_seed(5)
    params = [dict(temperature=t, top_p=p, repetition_penalty=1.3, presence_penalty=0.7,
                   frequency_penalty=0.2) for t, p in ((0.7, 0.9), (1.0, 0.5), (1.5, 0.95))]
    x = (torch.randn(len(params), V, generator=g) * 2.5).to(torch.bfloat16)
    rng = np.random.default_rng(6)
    rows = []
    for r in range(len(params)):
        top = torch.topk(x[r].float(), 200).indices.numpy()  # penalise the likely tokens
        rows.append(np.concatenate([top, rng.integers(0, V, 500)]))
    w = _workload(x, params, hist=_hist_csr(rows))
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])


@pytest.mark.parametrize("k", [40, 100, 150])
@pytest.mark.parametrize("batch,V", [(3, 151_936), (320, 20_000)])
def test_large_top_k_with_penalised_top_tokens(backend, k, batch, V):
    # rows with 32 < K <= 192 stream in a loop of their own (a running list of the K best
    # delegates); penalising the largest logits checks that delegates holding history ids never
    # lift the threshold. Three rows are cut into many runs; 320 rows share the CTAs.
    g = torch.Generator().manual_seed(1000 * k + batch)
    kinds = [dict(temperature=0.7, top_k=k, top_p=0.8, repetition_penalty=1.1,
                  presence_penalty=0.5, frequency_penalty=0.3),
             dict(temperature=1.0, top_k=k, repetition_penalty=1.5),
             dict(temperature=0.6, top_k=k, min_p=0.01, frequency_penalty=0.8)]
    params = [kinds[r % len(kinds)] for r in range(batch)]
    x = (torch.randn(batch, V, generator=g) * 2.0).to(torch.bfloat16)
    rng = np.random.default_rng(k + batch)
    rows = []
    for r in range(batch):
        top = torch.topk(x[r].float(), 2 * k).indices.numpy()
        rows.append(np.concatenate([top, rng.integers(0, V, 300)]))
    w = _workload(x, params, hist=_hist_csr(rows))
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    assert not rep.failures, (str(rep), rep.failures[:5])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_top_k_rows_with_penalties_that_raise_logits(backend, dtype):
    # repetition < 1 (or a negative presence / frequency penalty) lifts a penalised token, so
    # one whose raw logit was below the run's threshold can enter the top-k: these rows take the
    # gather of every penalised token at the run's end rather than the delegate expansion
    V = 40_000
    g = torch.Generator().manual_seed(21)
    kinds = [dict(temperature=0.8, top_k=20, top_p=0.9, repetition_penalty=0.7),
             dict(temperature=1.0, top_k=10, presence_penalty=-2.0),
             dict(temperature=0.6, top_k=32, top_p=0.8, frequency_penalty=-0.5),
             dict(temperature=1.0, top_k=5, repetition_penalty=0.8, presence_penalty=-1.0,
                  frequency_penalty=0.1)]
    params = kinds * 4
    B = len(params)
    x = (torch.randn(B, V, generator=g) * 2.0).to(dtype)
    rng = np.random.default_rng(5)
    ptr, ids_, cnt = [0], [], []
    for r in range(B):
        # tokens just below the top: penalties that raise them reorder the top-k
        order = torch.argsort(x[r].float(), descending=True).numpy()
        toks = np.concatenate([order[30:90], rng.integers(0, V, 100)])
        u, c = np.unique(toks, return_counts=True)
        ids_.append(u.astype(np.int32))
        cnt.append(c.astype(np.int32))
        ptr.append(ptr[-1] + len(u))
    w = _workload(x, params, hist=(np.array(ptr), np.concatenate(ids_), np.concatenate(cnt)))
    ids, probs = run_b200(backend, w)
    rep = compare(w, ids, probs)
    report(f"top-k rows with logit-raising penalties ({dtype})", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])


LOGPROB_ATOL = 2e-5  # natural-log units: float32 probabilities within 1e-5 relative, plus slack


@pytest.mark.parametrize("config,batch", [(2, 24), (3, 16), (5, 16)])
def test_logprobs_of_the_sampled_tokens(config, batch):
    # the sampled token's log-probability under the row's final distribution, against the
    # oracle's final probabilities; greedy rows have a one-hot distribution (log-probability 0)
    w = make(config, batch=batch)
    be = SAMPLER.resolve("b200", BackendContext(torch.device("cuda", 0), w.logits.dtype))
    lg, params, u, hist = to_device(w, be.device)
    lp = torch.empty(w.batch, dtype=torch.float32, device=be.device)
    ids = be.sample_batch(lg, params, u, hist, logprobs_out=lp).cpu().numpy()
    be.check()
    lp = lp.cpu().numpy()
    checked = 0
    for r in range(w.batch):
        res = oracle_row(w, r)
        if w.temperature[r] == 0:
            assert lp[r] == 0.0, (r, lp[r])
            continue
        if int(ids[r]) != res.token:
            assert res.boundary, (r, int(ids[r]), res.token)
            continue
        want = float(np.log(res.probs[res.token]))
        assert abs(float(lp[r]) - want) <= LOGPROB_ATOL, (r, float(lp[r]), want)
        checked += 1
    assert checked >= w.batch // 2


@pytest.mark.parametrize("config,batch,n", [(2, 24, 5), (3, 16, 20), (5, 16, 8)])
def test_top_logprobs(config, batch, n):
    # the n most likely tokens of each row's final distribution, in descending probability
    # (ties by ascending id), with their log-probabilities; tokens outside the kept set -inf
    w = make(config, batch=batch)
    be = SAMPLER.resolve("b200", BackendContext(torch.device("cuda", 0), w.logits.dtype))
    lg, params, u, hist = to_device(w, be.device)
    ids = be.sample_batch(lg, params, u, hist).cpu().numpy()
    tid, tlp = be.top_logprobs(lg, params, u, hist, n)
    be.check()
    tid, tlp = tid.cpu().numpy(), tlp.cpu().numpy()
    checked = 0
    for r in range(w.batch):
        res = oracle_row(w, r)
        if w.temperature[r] == 0:  # one-hot: the greedy token with log-probability 0
            assert tid[r, 0] == ids[r] and tlp[r, 0] == 0.0, (r, tid[r, :2], tlp[r, :2])
            assert np.all(np.isneginf(tlp[r, 1:])), (r, tlp[r])
            continue
        if res.boundary:
            continue
        if tid[r, 0] == -1:  # ties flooded the list (configuration 5's tied rows)
            continue
        p = res.probs
        kept = np.flatnonzero(p > 0)
        order = kept[np.lexsort((kept, -p[kept].astype(np.float64)))]
        m = min(n, len(order))
        assert tid[r, :m].tolist() == order[:m].tolist(), (r, tid[r, :m], order[:m])
        want = np.log(p[order[:m]].astype(np.float64))
        assert np.all(np.abs(tlp[r, :m] - want) <= LOGPROB_ATOL), (r, tlp[r, :m], want)
        assert np.all(np.isneginf(tlp[r, m:])), (r, tlp[r, m:])
        checked += 1
    assert checked >= w.batch // 3
