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


def test_noalloc_mixed_rows_coins_and_row_stride(pkg):
    """Greedy rows (T = 0), sample_mult rows (topp 0 or 1) and top-p rows in
    one batch, with drawn coins and then given coins, and a row stride
    ld > V: the same ids, states, probabilities and flags as sampler_batched
    on the same inputs."""
    L = _lib(pkg)
    B, V, ld = 96, 32000, 32008
    rng = np.random.default_rng(44)
    x = rng.normal(0, 2.0, (B, V)).astype(np.float32)
    temps = np.where(np.arange(B) % 4 == 0, 0.0, 0.8).astype(np.float32)
    topps = np.array([[0.9, 1.0, 0.0, 0.95][i % 4] for i in range(B)], np.float32)
    seeds = np.arange(B, dtype=np.uint64) * 5 + 1
    buf = torch.zeros(B, ld, device=DEV)
    buf[:, :V] = torch.from_numpy(x).to(DEV)
    xt = buf[:, :V]
    te = torch.from_numpy(temps).to(DEV)
    tp = torch.from_numpy(topps).to(DEV)
    for coins_np in (None, rng.random(B).astype(np.float32)):
        co = None if coins_np is None else torch.from_numpy(coins_np).to(DEV)
        res = []
        for noalloc in (True, False):
            st = torch.from_numpy(seeds.view(np.int64).copy()).to(DEV)
            ids = torch.full((B,), -1, dtype=torch.int32, device=DEV)
            probs = torch.empty(B, V, device=DEV)
            flags = torch.full((B,), -1, dtype=torch.int32, device=DEV)
            if noalloc:
                cfg = pkg.SamplerBatchConfig(V, 0.8, 0.9, 0)
                rc = L.sampler_batched_noalloc(ctypes.byref(cfg), _ptr(xt), B, ld, _ptr(te), _ptr(tp), _ptr(co),
                                               _ptr(st), _ptr(ids), _ptr(probs), _ptr(flags),
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
                assert rc == 0, rc
            else:
                pkg.sample_batched(xt, 0.8, 0.9, st, temperature_rows=te, topp_rows=tp, coins=co, out_ids=ids,
                                   probs_out=probs, row_flags=flags)
            torch.cuda.synchronize()
            res.append((ids.cpu().numpy(), st.cpu().numpy().view(np.uint64), probs.cpu().numpy(),
                        flags.cpu().numpy()))
        _same(*res)
        if coins_np is not None:  # given coins: the states are neither read nor written
            assert np.array_equal(res[0][1], seeds)


_FRESH_PROCESS = r"""
import ctypes, json, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from __graft_entry__ import load_package
pkg = load_package()
L = pkg.lib()
P = ctypes.c_void_p
L.sampler_batched_noalloc.argtypes = [ctypes.POINTER(pkg.SamplerBatchConfig), P, ctypes.c_int,
                                      ctypes.c_longlong, P, P, P, P, P, P, P, P]
B, V = 64, 32000
dev = torch.device("cuda:0")
w = pkg.workloads.topp(rows=B)
x = torch.from_numpy(w["logits"]).to(dev)
tr = torch.from_numpy(w["topp_rows"]).to(dev)
seeds = torch.from_numpy(pkg.workloads.row_seeds(B).view(np.int64).copy()).to(dev)
st = [seeds.clone() for _ in range(3)]
ids = [torch.empty(B, dtype=torch.int32, device=dev) for _ in range(3)]
cfg = pkg.SamplerBatchConfig(V, 0.7, 0.9, 0)
s = P(torch.cuda.current_stream().cuda_stream)
torch.cuda.synchronize()
free = []
for k in range(3):  # the library's first calls on this device: only the no-alloc entry point
    rc = L.sampler_batched_noalloc(ctypes.byref(cfg), P(x.data_ptr()), B, V, None, P(tr.data_ptr()), None,
                                   P(st[k].data_ptr()), P(ids[k].data_ptr()), None, None, s)
    assert rc == 0, rc
    torch.cuda.synchronize()
    free.append(torch.cuda.mem_get_info()[0])
same = all(torch.equal(ids[0], ids[k]) for k in range(3))
print(json.dumps(dict(free=free, same=same)))
"""


def test_noalloc_first_calls_allocate_nothing():
    """In a fresh process whose only library calls are to the no-alloc entry
    point: after the first call (which loads the library's device code and
    with it the fixed array), further calls leave the device's free memory
    unchanged."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, root], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["same"]
    assert out["free"][1] == out["free"][0] and out["free"][2] == out["free"][0], out["free"]


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
