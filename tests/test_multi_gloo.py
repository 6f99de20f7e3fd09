"""The row-sharded (N > 1) host logic, on CPU with gloo and world_size 2.

* Histogram words: every rank splits its exact partial sums into (hi, lo)
  int64 words; summing the words over ranks (all_reduce SUM, as NCCL does
  on the GPUs) recombines to exactly the single-process sum, for any row
  split.
* Global counts decide the smaller child and min_samples_leaf: the rank-local
  smaller side can differ from the global one.
* Row shards and the sampler: the ranks' contiguous row blocks cover every
  row once, and the union of the ranks' in-bag rows is the global draw.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shard(n, ws, rk):
    # the estimator's and bench.py's row blocks
    return (n * rk) // ws, (n * (rk + 1)) // ws


def _cells(q, bins, nb=16):
    """Exact per-bin sums of int64 q (Python ints, no overflow)."""
    out = [0] * nb
    for v, b in zip(q.tolist(), bins.tolist()):
        out[b] += int(v)
    return out


def _words(vals):
    hi = np.array([v >> 32 for v in vals], dtype=np.int64)
    lo = np.array([v & 0xFFFFFFFF for v in vals], dtype=np.int64)
    return hi, lo


def _worker(rank, ws, port, q, bins, go_left, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        n = len(q)
        lo_r, hi_r = _shard(n, ws, rank)
        local = _cells(q[lo_r:hi_r], bins[lo_r:hi_r])
        hi, lo = _words(local)
        t_hi, t_lo = torch.from_numpy(hi), torch.from_numpy(lo)
        dist.all_reduce(t_hi)
        dist.all_reduce(t_lo)
        total = [int(a) * (1 << 32) + int(b) for a, b in zip(t_hi.tolist(), t_lo.tolist())]
        nl = torch.tensor([int(go_left[lo_r:hi_r].sum())], dtype=torch.int64)
        local_left_small = bool(nl.item() <= (hi_r - lo_r) - nl.item())
        dist.all_reduce(nl)
        global_left_small = bool(nl.item() <= n - nl.item())
        result[rank] = (total, int(nl.item()), local_left_small, global_left_small)
    finally:
        dist.destroy_process_group()


def test_hist_words_sum_exactly_over_two_ranks():
    rng = np.random.default_rng(0)
    n = 4000
    S = 46
    g = rng.standard_normal(n) * 3.9
    q = np.rint(np.ldexp(g, S)).astype(np.int64)          # |q| < 2^48, like the engine
    bins = rng.integers(0, 16, n)
    # rows of rank 0 mostly go left, rank 1's mostly right: local and global
    # smaller sides disagree on one rank
    go_left = np.concatenate([rng.random(n // 2) < 0.9, rng.random(n - n // 2) < 0.3])
    mgr = mp.Manager()
    result = mgr.dict()
    port = _free_port()
    mp.spawn(_worker, args=(2, port, q, bins, go_left, result), nprocs=2, join=True)
    want = _cells(q, bins)
    for rk in range(2):
        total, gl, _, gsmall = result[rk]
        assert total == want
        assert gl == int(go_left.sum())
        assert gsmall == bool(go_left.sum() <= n - go_left.sum())
    # every rank takes the global decision, even where its own rows disagree
    assert result[0][3] == result[1][3]
    assert result[0][2] != result[1][2]


@pytest.mark.parametrize("n,ws", [(10, 2), (1_000_001, 8), (7, 8), (12345, 3)])
def test_row_shards_cover_every_row_once(n, ws):
    seen = np.zeros(n, dtype=np.int64)
    for rk in range(ws):
        lo, hi = _shard(n, ws, rk)
        seen[lo:hi] += 1
    assert np.all(seen == 1)


def test_sampler_union_of_rank_masks_is_the_global_draw(built_lib):
    from bsscl_gbm_b200 import Sampler
    n, p, ws = 10_001, 12, 4
    s = Sampler(9, n, p, int(n * 0.75), 8, True, True)
    smp, mask, feat = s.next(want_sample=True, want_mask=True)
    s.close()
    union = np.zeros(n, dtype=np.uint8)
    for rk in range(ws):
        lo, hi = _shard(n, ws, rk)
        union[lo:hi] = mask[lo:hi]                         # what rank rk uploads
    assert np.array_equal(np.nonzero(union)[0], np.sort(smp))


def _predict_worker(rank, ws, port, n, result):
    """Row-sharded predict's host logic: each rank scores only its own block
    (here a stand-in score: the row index itself) and _gather_rows returns
    every row, in order, on every rank."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from bsscl_gbm_b200.estimator import _gather_rows, _rank_rows
        lo, hi = _rank_rows(n)
        local = np.stack([np.arange(lo, hi, dtype=np.float64), -np.arange(lo, hi, dtype=np.float64)], axis=1)
        result[rank] = (lo, hi, _gather_rows(dist, local, n))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [11, 4000])
def test_sharded_predict_gathers_every_row_in_order(n):
    mgr = mp.Manager()
    result = mgr.dict()
    mp.spawn(_predict_worker, args=(2, _free_port(), n, result), nprocs=2, join=True)
    want = np.stack([np.arange(n, dtype=np.float64), -np.arange(n, dtype=np.float64)], axis=1)
    assert result[0][:2] == (0, n // 2) and result[1][:2] == (n // 2, n)
    for rk in range(2):
        assert np.array_equal(result[rk][2], want)
