"""GPU: the allocation-free batched entry point.

Callers whose device memory belongs to another allocator (an inference
server's arena, a framework's caching allocator) or that must not let
cudaMalloc/cudaFree synchronize the device cannot use sampler_batched's
library-managed workspace.  sampler_batched_noalloc runs the same kernel with
its scratch in an array compiled into the library.  This file is collected
last on purpose: it calls the new entry point through the C-ABI, twice in a
row with different inputs (the second call reuses the shared array after the
first left its contents there), and checks each result against the regular
entry point on the same inputs, within the tolerances of the parity tests.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-6
DEV = torch.device("cuda:0")


def _lib(pkg):
    L = pkg.lib()
    P = ctypes.c_void_p
    L.sampler_batched_noalloc.argtypes = [ctypes.POINTER(pkg.SamplerBatchConfig), P, ctypes.c_int,
                                          ctypes.c_longlong, P, P, P, P, P, P, P, P]
    L.sampler_batched_noalloc.restype = ctypes.c_int
    return L


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(x, seeds, topp_rows):
    xt = torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    st = torch.from_numpy(np.asarray(seeds, np.uint64).view(np.int64).copy()).to(DEV)
    tr = None if topp_rows is None else torch.from_numpy(np.asarray(topp_rows, np.float32)).to(DEV)
    return xt, st, tr


def run_noalloc(pkg, x, temp, topp, seeds, topp_rows=None):
    L = _lib(pkg)
    B, V = x.shape
    xt, st, tr = _inputs(x, seeds, topp_rows)
    ids = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    probs = torch.empty(B, V, device=DEV)
    flags = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    cfg = pkg.SamplerBatchConfig(V, temp, topp, 0)
    rc = L.sampler_batched_noalloc(ctypes.byref(cfg), _ptr(xt), B, V, None, _ptr(tr), None, _ptr(st), _ptr(ids),
                                   _ptr(probs), _ptr(flags), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()
    return ids.cpu().numpy(), st.cpu().numpy().view(np.uint64), probs.cpu().numpy(), flags.cpu().numpy()


def run_regular(pkg, x, temp, topp, seeds, topp_rows=None):
    B, V = x.shape
    xt, st, tr = _inputs(x, seeds, topp_rows)
    probs = torch.empty(B, V, device=DEV)
    flags = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    ids = pkg.sample_batched(xt, temp, topp, st, topp_rows=tr, probs_out=probs, row_flags=flags)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), st.cpu().numpy().view(np.uint64), probs.cpu().numpy(), flags.cpu().numpy()


def _same(a, b):
    ids_a, st_a, p_a, f_a = a
    ids_b, st_b, p_b, f_b = b
    assert np.array_equal(ids_a, ids_b)
    assert np.array_equal(st_a, st_b)
    assert np.array_equal(f_a, f_b)
    pos = p_b > 0
    rel = np.abs(p_a[pos].astype(np.float64) - p_b[pos]) / p_b[pos]
    assert (rel.max() if rel.size else 0.0) <= PROB_RTOL
    assert np.all(p_a[~pos] == p_b[~pos])


def test_noalloc_matches_batched_entry_point_two_calls(pkg):
    w = pkg.workloads.topp(rows=300)
    seeds = pkg.workloads.row_seeds(300)
    # call 1: ordinary top-p rows
    _same(run_noalloc(pkg, w["logits"], 0.7, 0.9, seeds, w["topp_rows"]),
          run_regular(pkg, w["logits"], 0.7, 0.9, seeds, w["topp_rows"]))
    # call 2: flat rows whose nucleus takes the slow path through the scratch
    flat = np.random.default_rng(15).normal(0, 0.05, (40, 32000)).astype(np.float32)
    s2 = np.arange(40, dtype=np.uint64) + 100
    got = run_noalloc(pkg, flat, 1.0, 0.95, s2)
    assert (got[3] & pkg.ROW_SLOW_PATH).all()
    _same(got, run_regular(pkg, flat, 1.0, 0.95, s2))


def test_noalloc_rejects_vocab_above_limit(pkg):
    L = _lib(pkg)
    V = 32768 + 4
    x = torch.zeros(2, V, device=DEV)
    ids = torch.empty(2, dtype=torch.int32, device=DEV)
    st = torch.zeros(2, dtype=torch.int64, device=DEV)
    cfg = pkg.SamplerBatchConfig(V, 1.0, 0.9, 0)
    rc = L.sampler_batched_noalloc(ctypes.byref(cfg), _ptr(x), 2, V, None, None, None, _ptr(st), _ptr(ids), None,
                                   None, None)
    assert rc == -2  # SAMPLER_E_UNSUPPORTED
