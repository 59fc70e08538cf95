"""GPU: failure detection and concurrency of the library-managed buffers.

* A bounded device wait that runs out is reported, not hung on: the
  self-test entry point makes the row kernel's first wait run out on a barrier
  that no copy targets (nothing is left in flight), and the status comes back
  as SAMPLER_E_DEVICE with the row flagged SAMPLER_ROW_TIMEOUT; the next call
  on the device runs normally.  No GPU fault is involved.
* Calls on different streams with the library-managed workspace may overlap:
  each stream has its own workspace, so concurrent calls give the results
  each gives alone.
"""
import ctypes

import numpy as np
import pytest
import torch

from test_gpu_parity import check_e2e, gpu_sample

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
SAMPLER_E_DEVICE = -6


def test_bounded_wait_timeout_is_reported(pkg, orc):
    L = pkg.lib()
    flag = ctypes.c_int(-1)
    rc = L.sampler_selftest_wait_timeout(1 << 12, ctypes.byref(flag))
    assert rc == SAMPLER_E_DEVICE, L.sampler_last_error()
    assert flag.value == pkg.ROW_TIMEOUT
    assert b"bounded device wait" in L.sampler_last_error()
    # the context stays usable and the error word was cleared
    w = pkg.workloads.topp(rows=64)
    seeds = pkg.workloads.row_seeds(64)
    out = gpu_sample(pkg, w["logits"], 0.7, 0.9, seeds=seeds, topp_rows=w["topp_rows"])
    ref_ids, ref_st, ref_p = orc.sample_batch(w["logits"], 0.7, 0.9, seeds, topp_rows=w["topp_rows"], probs_out=True)
    assert np.array_equal(out["states"], ref_st) and (out["flags"] & pkg.ROW_TIMEOUT == 0).all()
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, w["topp_rows"])
    # a synchronous entry point sees no stale error
    s = pkg.build_sampler(32000, 0.7, 0.9, 42)
    assert pkg.sample(s, w["logits"][0].copy()) >= 0
    pkg.free_sampler(s)


def test_selftest_rejects_bad_arguments(pkg):
    L = pkg.lib()
    flag = ctypes.c_int(0)
    assert L.sampler_selftest_wait_timeout(0, ctypes.byref(flag)) == -1
    assert L.sampler_selftest_wait_timeout(16, None) == -1


def _run(pkg, x, temp, topp, seeds, stream, topp_rows=None):
    xt = torch.from_numpy(x).to(DEV)
    st = torch.from_numpy(seeds.view(np.int64).copy()).to(DEV)
    tr = None if topp_rows is None else torch.from_numpy(topp_rows).to(DEV)
    flags = torch.full((x.shape[0],), -1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    return xt, st, tr, flags


def test_two_streams_with_library_workspace(pkg, orc):
    """Top-p rows on one stream and flat rows (nuclei through the L2 scratch
    of the workspace, the deferred-row list) on another, issued back to back
    several times so the calls overlap; every result equals the same call
    made alone."""
    w = pkg.workloads.topp(rows=600)
    x1, tr1 = w["logits"], w["topp_rows"]
    s1 = pkg.workloads.row_seeds(600)
    x2 = np.random.default_rng(15).normal(0, 0.05, (160, 32000)).astype(np.float32)
    s2 = np.arange(160, dtype=np.uint64) + 100
    # alone
    a1 = gpu_sample(pkg, x1, 0.7, 0.9, seeds=s1, topp_rows=tr1)
    a2 = gpu_sample(pkg, x2, 1.0, 0.95, seeds=s2)
    assert (a2["flags"] & pkg.ROW_SLOW_PATH).all()
    # together, on two streams
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    in1 = _run(pkg, x1, 0.7, 0.9, s1, streams[0], tr1)
    in2 = _run(pkg, x2, 1.0, 0.95, s2, streams[1])
    outs = []
    for rep in range(4):
        st1, st2 = in1[1].clone(), in2[1].clone()
        torch.cuda.synchronize()
        ids1 = pkg.sample_batched(in1[0], 0.7, 0.9, st1, topp_rows=in1[2], row_flags=in1[3], stream=streams[0])
        ids2 = pkg.sample_batched(in2[0], 1.0, 0.95, st2, row_flags=in2[3], stream=streams[1])
        outs.append((ids1, st1, ids2, st2))
    torch.cuda.synchronize()
    for ids1, st1, ids2, st2 in outs:
        assert np.array_equal(ids1.cpu().numpy(), a1["ids"])
        assert np.array_equal(st1.cpu().numpy().view(np.uint64), a1["states"])
        assert np.array_equal(ids2.cpu().numpy(), a2["ids"])
        assert np.array_equal(st2.cpu().numpy().view(np.uint64), a2["states"])
    # and against the oracle
    ref_ids, ref_st, ref_p = orc.sample_batch(x2, 1.0, 0.95, s2, probs_out=True)
    assert np.array_equal(a2["states"], ref_st)
    check_e2e(orc, a2["ids"], ref_ids, ref_p, s2, np.full(160, 0.95))
