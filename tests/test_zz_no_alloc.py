"""gbm_predict_noalloc: the predict entry point that allocates nothing.

It serves callers that cannot call cudaMalloc (a serving process that hands
out GPU memory from its own arena, a framework owning the device, a
latency-bound path where an allocation may synchronise the device).  The
caller owns every input and output buffer; the library's only scratch is a
fixed device array.  This test allocates the caller's buffers with torch,
calls the entry point through the C ABI twice in a row with different
ensembles (the shared scratch must not leak the first call's contents into
the second), and compares with gbm_predict, which stages the ensemble in
context-allocated memory.  The file is collected last so a failure here
comes after every other test has run.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _call(L, torch, xb_t, p, ens, n_trees, lr, base, stream):
    n = xb_t.shape[0]
    t = {k: _dev(torch, v) for k, v in ens.items()}
    F = torch.empty(n, dtype=torch.float64, device="cuda")
    P = torch.empty(n, dtype=torch.float64, device="cuda")
    err = C.create_string_buffer(256)
    rc = L.gbm_predict_noalloc(
        C.c_void_p(xb_t.data_ptr()), n, p, C.c_void_p(t["features"].data_ptr()),
        C.c_void_p(t["thresholds"].data_ptr()), C.c_void_p(t["values"].data_ptr()),
        C.c_void_p(t["left"].data_ptr()), C.c_void_p(t["right"].data_ptr()),
        C.c_void_p(t["offsets"].data_ptr()), n_trees, int(ens["features"].shape[0]), lr, base,
        C.c_void_p(F.data_ptr()), C.c_void_p(P.data_ptr()), stream, err, 256)
    return rc, err.value.decode(), F, P


def _ensemble(seed, n_trees, depth, p):
    from bsscl_gbm_b200 import datasets as D
    e = D.config5_ensemble(n_trees=n_trees, depth=depth, p=p, seed=seed)
    return {"features": e["features"].astype(np.int16), "thresholds": e["thresholds"].astype(np.int64),
            "values": e["values"].astype(np.float64), "left": e["left"].astype(np.int32),
            "right": e["right"].astype(np.int32), "offsets": e["offsets"].astype(np.int32)}


def test_predict_noalloc_matches_predict_twice():
    import torch
    from bsscl_gbm_b200 import Engine, lib
    L = lib()
    rng = np.random.default_rng(11)
    n, p = 20_000, 24
    xb = rng.integers(0, 256, size=(n, p)).astype(np.uint8)
    xb_t = _dev(torch, xb)
    eng = Engine(0)
    cases = [(_ensemble(3, 50, 8, p), 50, 0.08, -1.25, None),
             (_ensemble(4, 7, 5, p), 7, 0.3, 0.5, torch.cuda.current_stream().cuda_stream)]
    for ens, T, lr, base, stream in cases:
        rc, msg, F, P = _call(L, torch, xb_t, p, ens, T, lr, base, stream)
        assert rc == 0, msg
        F_ref, P_ref = eng.predict(xb, ens, T, lr, base)
        assert np.abs(F.cpu().numpy() - F_ref).max() <= 1e-12
        assert np.abs(P.cpu().numpy() - P_ref).max() <= 1e-12
    eng.close()


def test_predict_noalloc_allocates_nothing():
    """After a first call (which looks up the scratch array's address and
    loads the kernels), a second call leaves the device's free memory
    exactly as it was: every buffer it touches is the caller's or the fixed
    array."""
    import torch
    from bsscl_gbm_b200 import lib
    L = lib()
    rng = np.random.default_rng(12)
    n, p = 30_000, 16
    xb_t = _dev(torch, rng.integers(0, 256, size=(n, p)).astype(np.uint8))
    ens = _ensemble(7, 40, 7, p)
    t = {k: _dev(torch, v) for k, v in ens.items()}
    F = torch.empty(n, dtype=torch.float64, device="cuda")
    P = torch.empty(n, dtype=torch.float64, device="cuda")
    err = C.create_string_buffer(256)

    def call():
        return L.gbm_predict_noalloc(
            C.c_void_p(xb_t.data_ptr()), n, p, C.c_void_p(t["features"].data_ptr()),
            C.c_void_p(t["thresholds"].data_ptr()), C.c_void_p(t["values"].data_ptr()),
            C.c_void_p(t["left"].data_ptr()), C.c_void_p(t["right"].data_ptr()),
            C.c_void_p(t["offsets"].data_ptr()), 40, int(ens["features"].shape[0]), 0.1, 0.0,
            C.c_void_p(F.data_ptr()), C.c_void_p(P.data_ptr()), None, err, 256)

    assert call() == 0, err.value
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    assert call() == 0, err.value
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_predict_noalloc_rejects_oversize_and_malformed():
    import torch
    from bsscl_gbm_b200 import lib
    L = lib()
    n, p = 1000, 8
    xb_t = _dev(torch, np.zeros((n, p), np.uint8))
    big = _ensemble(5, 1100, 8, p)            # 562,100 nodes > 524,288
    rc, msg, _, _ = _call(L, torch, xb_t, p, big, 1100, 0.1, 0.0, None)
    assert rc == 1 and "524288 nodes" in msg
    many = _ensemble(8, 70_000, 0, p)          # 70,000 one-leaf trees > 65,536
    rc, msg, _, _ = _call(L, torch, xb_t, p, many, 70_000, 0.1, 0.0, None)
    assert rc == 1 and "65536 trees" in msg
    bad = _ensemble(6, 3, 3, p)
    bad["left"][0] = 0                         # a child that is not after its parent
    rc, msg, _, _ = _call(L, torch, xb_t, p, bad, 3, 0.1, 0.0, None)
    assert rc == 1 and "malformed" in msg
