"""Slotted decode histories on CPU: the host layout the device kernels and the sampler rely on
(ids ascending within a slot, padding above every vocabulary id with count 0), and a host model
of one append step that the GPU tests check the kernel against."""

from __future__ import annotations

import numpy as np
import pytest

from vinfer_b200.sampling import HIST_PAD_ID, SlotHistogram


def append_model(slots: list[dict[int, int]], tokens, cap: int) -> bool:
    """One vinfer_hist_append step on host dicts; returns whether some slot was full."""
    full = False
    for s, t in enumerate(tokens):
        t = int(t)
        if t < 0:
            continue
        if t in slots[s]:
            slots[s][t] += 1
        elif len(slots[s]) >= cap:
            full = True
        else:
            slots[s][t] = 1
    return full


def test_host_layout_is_a_valid_csr_history():
    rows = [[5, 3, 5, 9], [], [7] * 4, list(range(8))]
    cap = 8
    ids, counts, lens = SlotHistogram.host_layout(rows, cap)
    assert ids.dtype == np.int32 and counts.dtype == np.int32 and lens.dtype == np.int32
    assert lens.tolist() == [3, 0, 1, 8]
    for s in range(len(rows)):
        seg = ids[s * cap:(s + 1) * cap].astype(np.int64)
        assert np.all(seg[1:] > seg[:-1]), "ids ascend within a slot, padding included"
        assert np.all(counts[s * cap + lens[s]:(s + 1) * cap] == 0)
        assert np.all(seg[lens[s]:] > 262144), "padding lies above every vocabulary id"
        u, c = np.unique(np.asarray(rows[s], np.int64), return_counts=True)
        assert seg[:lens[s]].tolist() == u.tolist()
        assert counts[s * cap:s * cap + lens[s]].tolist() == c.tolist()
    # padding of position p: HIST_PAD_ID - (cap - 1 - p)
    assert ids[cap - 1] == HIST_PAD_ID and ids[1 * cap] == HIST_PAD_ID - (cap - 1)


def test_host_layout_rejects_overfull_slots_and_bad_ids():
    with pytest.raises(ValueError, match="more than cap"):
        SlotHistogram.host_layout([[1, 2, 3]], 2)
    with pytest.raises(ValueError, match="outside the vocabulary"):
        SlotHistogram.host_layout([[-1]], 4)


def test_append_model():
    slots = [{3: 1}, {}, {1: 1, 2: 1}]
    full = append_model(slots, [3, -1, 4], cap=2)
    assert slots == [{3: 2}, {}, {1: 1, 2: 1}] and full


def test_slots_from_csr_match_slots_from_token_lists():
    rng = np.random.default_rng(2)
    rows = [rng.integers(0, 500, rng.integers(0, 60)).tolist() for _ in range(7)]
    a = SlotHistogram.from_token_lists(rows, 64, "cpu")
    ptr, ids, cnt = [0], [], []
    for toks in rows:
        u, c = np.unique(np.asarray(toks, np.int64), return_counts=True)
        ids.append(u.astype(np.int32))
        cnt.append(c.astype(np.int32))
        ptr.append(ptr[-1] + len(u))
    b = SlotHistogram.from_csr(np.array(ptr), np.concatenate(ids), np.concatenate(cnt), 64, "cpu")
    for name in ("ids", "counts", "lens", "row_ptr"):
        assert np.array_equal(getattr(a, name).numpy(), getattr(b, name).numpy()), name
    assert a.to_counts() == b.to_counts()
    assert b.history.row_ptr.tolist() == [64 * s for s in range(8)]
