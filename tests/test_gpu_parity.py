"""GPU parity of the sm_100a sampler against the oracle and the golden ids of
the reference's own sampler.  Every call goes through the C-ABI library.

Bars (from the llama2.c Sampler contract):
  * argmax ids: bit-exact;
  * given the reference's fp32 probabilities (PROBS_IN), sample_mult and
    sample_topp ids: bit-exact;
  * end to end from logits: probabilities within PROB_RTOL relative, ids
    matching on >= 99.99% of rows, and every mismatch attributable to a coin
    within BOUNDARY of a cdf boundary of the reference's walk;
  * xorshift states after the call: bit-exact.
"""
import ctypes
import hashlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-6      # relative tolerance on probabilities (end to end)
BOUNDARY = 1e-6       # a mismatching id must come from a coin this close to a cdf value
MIN_MATCH = 0.9999    # fraction of ids that must match end to end

DEV = torch.device("cuda:0")


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def gpu_sample(pkg, x, temp, topp, seeds=None, topp_rows=None, temp_rows=None, coins=None, probs_in=False,
               want_probs=False, ld=None, mode=0):
    B, V = x.shape
    if ld is not None and ld != V:
        buf = torch.zeros(B, ld, device=DEV)
        buf[:, :V] = torch.from_numpy(x).to(DEV)
        xt = buf[:, :V]
    else:
        xt = torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    st = None if seeds is None else torch.from_numpy(np.asarray(seeds, np.uint64).view(np.int64).copy()).to(DEV)
    tr = None if topp_rows is None else torch.from_numpy(np.asarray(topp_rows, np.float32)).to(DEV)
    te = None if temp_rows is None else torch.from_numpy(np.asarray(temp_rows, np.float32)).to(DEV)
    co = None if coins is None else torch.from_numpy(np.asarray(coins, np.float32)).to(DEV)
    probs = torch.empty(B, V, device=DEV) if want_probs else None
    flags = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    ids = pkg.sample_batched(xt, temp, topp, st, topp_rows=tr, temperature_rows=te, coins=co, probs_out=probs,
                             row_flags=flags, probs_in=probs_in, mode=mode)
    torch.cuda.synchronize()
    out = dict(ids=ids.cpu().numpy(), flags=flags.cpu().numpy())
    if st is not None:
        out["states"] = st.cpu().numpy().view(np.uint64)
    if want_probs:
        out["probs"] = probs.cpu().numpy()
    return out


def prob_rel_err(p, ref):
    pos = ref > 0
    rel = np.abs(p[pos].astype(np.float64) - ref[pos]) / ref[pos]
    zero_ok = np.all(np.abs(p[~pos]) <= 1e-37) if (~pos).any() else True
    return (float(rel.max()) if rel.size else 0.0), bool(zero_ok)


def check_e2e(orc, got, ref_ids, ref_probs, seeds, topps):
    if len(ref_ids) == 0:
        return 0
    mism = np.nonzero(got != ref_ids)[0]
    assert 1.0 - len(mism) / len(ref_ids) >= MIN_MATCH, f"{len(mism)} mismatching ids of {len(ref_ids)}"
    for r in mism:
        coin, _ = orc.coin(int(seeds[r]))
        d = orc.boundary_distance(ref_probs[r], float(topps[r]), coin)
        assert d <= BOUNDARY, f"row {r}: id {got[r]} vs {ref_ids[r]} with the coin {d:.3g} from any boundary"
    return len(mism)


# ---------------------------------------------------------------------------
def test_argmax_workload_bit_exact(pkg, golden):
    w = pkg.workloads.argmax()
    out = gpu_sample(pkg, w["logits"], 0.0, 0.9)
    assert out["ids"].tolist() == golden["argmax"]["ids"]
    assert (out["flags"] == 0).all()


def test_argmax_in_row_kernel_bit_exact(pkg, golden):
    """Greedy rows mixed into a sampling batch (per-row temperature) take the
    row kernel's argmax; same ids."""
    w = pkg.workloads.argmax()
    temps = np.zeros(256, np.float32)
    out = gpu_sample(pkg, w["logits"], 0.8, 0.9, seeds=np.arange(256, dtype=np.uint64), temp_rows=temps)
    assert out["ids"].tolist() == golden["argmax"]["ids"]
    assert np.array_equal(out["states"], np.arange(256, dtype=np.uint64))  # no draw on greedy rows


@pytest.mark.parametrize("rows", [[np.nan, 1.0, 2.0, 2.0], [1.0, np.nan, 2.0, 2.0], [-0.0, 0.0, -1.0, -2.0],
                                  [-np.inf, -np.inf, -np.inf, -np.inf], [np.nan] * 4, [1.0, np.inf, np.inf, 3.0]])
def test_argmax_special_values(pkg, orc, rows):
    x = np.tile(np.array(rows, np.float32), (3, 1))
    out = gpu_sample(pkg, x, 0.0, 0.9)
    assert out["ids"].tolist() == [orc.argmax(r) for r in x]


def test_probs_in_bit_exact(pkg, orc, golden):
    wl = pkg.workloads
    g = golden["probs_in"]
    _, _, pm = orc.sample_batch(wl.mult(rows=256)["logits"], 0.8, 1.0, wl.row_seeds(256), probs_out=True)
    w = wl.topp(rows=256)
    _, _, pt = orc.sample_batch(w["logits"], 0.7, 0.9, wl.row_seeds(256), topp_rows=w["topp_rows"], probs_out=True)
    assert digest(pm) == g["mult_probs_sha"] and digest(pt) == g["topp_probs_sha"], \
        "host expf differs from the fixture's: the oracle does not reproduce the reference probabilities here"
    om = gpu_sample(pkg, pm, 1.0, 1.0, seeds=wl.row_seeds(256), probs_in=True)
    assert om["ids"].tolist() == g["mult_ids"]
    ot = gpu_sample(pkg, pt, 1.0, 0.9, seeds=wl.row_seeds(256), topp_rows=w["topp_rows"], probs_in=True)
    assert ot["ids"].tolist() == g["topp_ids"]
    _, st = orc.sample_probs_batch(pt, 0.9, wl.row_seeds(256), topp_rows=w["topp_rows"])
    assert np.array_equal(ot["states"], st)


def test_probs_in_random_bit_exact(pkg, orc):
    """Given probabilities and coins, ids equal the oracle's sample_mult /
    sample_topp for many shapes of distribution."""
    rng = np.random.default_rng(21)
    for V, sigma, topp in [(32000, 2.0, 0.9), (32000, 0.3, 0.95), (32000, 6.0, 0.5), (5003, 1.0, 0.9),
                           (32000, 1.0, 1.0), (129, 3.0, 0.7)]:
        x = rng.normal(0, sigma, (64, V)).astype(np.float32)
        _, _, p = orc.sample_batch(x, 1.0, 0.5, np.zeros(64, np.uint64), probs_out=True)
        coins = rng.random(64).astype(np.float32)
        out = gpu_sample(pkg, p, 1.0, topp, coins=coins, probs_in=True)
        want = [orc.mult(p[r], coins[r]) if topp >= 1.0 else orc.topp(p[r], topp, coins[r]) for r in range(64)]
        assert out["ids"].tolist() == want, (V, sigma, topp)


def test_mult_workload_end_to_end(pkg, orc, golden):
    w = pkg.workloads.mult()
    seeds = pkg.workloads.row_seeds(1024)
    out = gpu_sample(pkg, w["logits"], w["temperature"], w["topp"], seeds=seeds, want_probs=True)
    ref_ids, ref_st, ref_p = orc.sample_batch(w["logits"], w["temperature"], w["topp"], seeds, probs_out=True)
    assert ref_ids.tolist() == golden["mult"]["ids"]
    rel, zero_ok = prob_rel_err(out["probs"], ref_p)
    assert rel <= PROB_RTOL and zero_ok, rel
    assert np.array_equal(out["states"], ref_st)
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, np.ones(1024))


def test_mult_workload_streamed(pkg, orc, golden):
    """Without probability write-back, sample_mult rows take the streaming
    kernel's cdf walk (chunk functions of the exact p's)."""
    w = pkg.workloads.mult()
    seeds = pkg.workloads.row_seeds(1024)
    out = gpu_sample(pkg, w["logits"], w["temperature"], w["topp"], seeds=seeds)
    ref_ids, ref_st, ref_p = orc.sample_batch(w["logits"], w["temperature"], w["topp"], seeds, probs_out=True)
    assert ref_ids.tolist() == golden["mult"]["ids"]
    assert np.array_equal(out["states"], ref_st)
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, np.ones(1024))
    small = out["ids"][:64]  # the 1024-thread shape (batch below the SM count) on the same rows
    out64 = gpu_sample(pkg, w["logits"][:64], w["temperature"], w["topp"], seeds=seeds[:64])
    assert np.array_equal(out64["ids"], small)


def test_topp_workload_end_to_end(pkg, orc, golden):
    w = pkg.workloads.topp()
    seeds = pkg.workloads.row_seeds(4096)
    out = gpu_sample(pkg, w["logits"], w["temperature"], w["topp"], seeds=seeds, topp_rows=w["topp_rows"],
                     want_probs=True)
    ref_ids, ref_st, ref_p = orc.sample_batch(w["logits"], w["temperature"], w["topp"], seeds,
                                              topp_rows=w["topp_rows"], probs_out=True)
    assert ref_ids.tolist() == golden["topp"]["ids"]
    rel, zero_ok = prob_rel_err(out["probs"], ref_p)
    assert rel <= PROB_RTOL and zero_ok, rel
    assert np.array_equal(out["states"], ref_st)
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, w["topp_rows"])


def test_topp_workload_pipelined_path(pkg, orc, golden):
    """Without probability write-back the batch takes the pipelined kernel
    (rows it defers finish in the general kernel)."""
    w = pkg.workloads.topp()
    seeds = pkg.workloads.row_seeds(4096)
    out = gpu_sample(pkg, w["logits"], w["temperature"], w["topp"], seeds=seeds, topp_rows=w["topp_rows"])
    ref_ids, ref_st, ref_p = orc.sample_batch(w["logits"], w["temperature"], w["topp"], seeds,
                                              topp_rows=w["topp_rows"], probs_out=True)
    assert np.array_equal(out["states"], ref_st)
    assert (out["flags"] >= 0).all()
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, w["topp_rows"])


def test_mixed_modes_in_one_batch(pkg, orc):
    """Greedy, top-p and multinomial rows together (per-row temperature and
    topp), all on the streaming kernel."""
    rng = np.random.default_rng(41)
    B = 300
    x = rng.normal(0, 2.5, (B, 32000)).astype(np.float32)
    temps = np.where(np.arange(B) % 5 == 0, 0.0, 0.9).astype(np.float32)
    topps = np.where(np.arange(B) % 3 == 0, 1.0, 0.9).astype(np.float32)
    seeds = np.arange(B, dtype=np.uint64) * 7 + 3
    out = gpu_sample(pkg, x, 0.9, 0.9, seeds=seeds, topp_rows=topps, temp_rows=temps)
    ids, states = [], []
    for r in range(B):
        i, s_ = orc.sample_batch(x[r:r + 1], float(temps[r]), float(topps[r]), seeds[r:r + 1])
        ids.append(int(i[0]))
        states.append(int(s_[0]))
    assert np.array_equal(out["states"], np.array(states, np.uint64))
    mism = [r for r in range(B) if out["ids"][r] != ids[r]]
    for r in mism:
        _, _, rp = orc.sample_batch(x[r:r + 1], float(temps[r]), float(topps[r]), seeds[r:r + 1], probs_out=True)
        coin, _ = orc.coin(int(seeds[r]))
        assert temps[r] != 0.0 and orc.boundary_distance(rp[0], float(topps[r]), coin) <= BOUNDARY


def test_large_nucleus_deferred_from_pipeline(pkg, orc):
    x = np.random.default_rng(15).normal(0, 0.05, (8, 32000)).astype(np.float32)
    seeds = np.arange(8, dtype=np.uint64) + 100
    out = gpu_sample(pkg, x, 1.0, 0.95, seeds=seeds)
    assert (out["flags"] & pkg.ROW_SLOW_PATH).all()
    ref_ids, ref_st, ref_p = orc.sample_batch(x, 1.0, 0.95, seeds, probs_out=True)
    assert np.array_equal(out["states"], ref_st)
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, np.full(8, 0.95))


@pytest.mark.parametrize("sigma,temp,topp", [(1.6, 0.8, 0.9), (1.0, 1.0, 0.99), (2.5, 0.7, 0.5), (1.2, 0.9, 0.95)])
def test_large_nucleus_fast_path(pkg, orc, sigma, temp, topp):
    """Nuclei of hundreds to thousands of tokens stay in the streaming kernel
    (the cumulative walk by chunk functions) and match the oracle."""
    x = np.random.default_rng(23).normal(0, sigma, (64, 32000)).astype(np.float32)
    seeds = np.arange(64, dtype=np.uint64) + 500
    out = gpu_sample(pkg, x, temp, topp, seeds=seeds)
    assert not (out["flags"] & pkg.ROW_SLOW_PATH).any()
    ref_ids, ref_st, ref_p = orc.sample_batch(x, temp, topp, seeds, probs_out=True)
    assert np.array_equal(out["states"], ref_st)
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, np.full(64, topp))


def test_topp_without_probability_writeback_same_ids(pkg):
    """The fast path (no probs_out) computes p only for candidates; ids must
    not change."""
    w = pkg.workloads.topp(rows=512)
    seeds = pkg.workloads.row_seeds(512)
    a = gpu_sample(pkg, w["logits"], 0.7, 0.9, seeds=seeds, topp_rows=w["topp_rows"], want_probs=True)
    b = gpu_sample(pkg, w["logits"], 0.7, 0.9, seeds=seeds, topp_rows=w["topp_rows"])
    assert np.array_equal(a["ids"], b["ids"]) and np.array_equal(a["states"], b["states"])


def test_single_row_sampler_api(pkg, orc, golden):
    """llama2.c drop-in: one Sampler seeded 42, sample() over 256 rows."""
    w = pkg.workloads.single_row()
    s = pkg.build_sampler(32000, w["temperature"], w["topp"], w["seed"])
    ids = []
    probs = []
    for r in range(256):
        row = w["logits"][r].copy()
        ids.append(pkg.sample(s, row))
        probs.append(row)
    state = s.rng_state
    pkg.free_sampler(s)
    g = golden["single_row"]["ids"]
    st = 42
    for r in range(256):
        coin, st = orc.coin(st)
        if ids[r] != g[r]:
            ref_row = w["logits"][r].copy()
            _, _, rp = orc.sample_batch(ref_row[None, :], w["temperature"], w["topp"], np.zeros(1, np.uint64),
                                        probs_out=True)
            assert orc.boundary_distance(rp[0], w["topp"], coin) <= BOUNDARY
    assert state == st
    # sample() leaves the probabilities in the caller's buffer
    _, _, rp = orc.sample_batch(w["logits"][:4], w["temperature"], w["topp"], np.zeros(4, np.uint64), probs_out=True)
    rel, _ = prob_rel_err(np.stack(probs[:4]), rp)
    assert rel <= PROB_RTOL


def test_direct_entry_points(pkg, orc):
    L = pkg.lib()
    rng = np.random.default_rng(31)
    x = rng.normal(0, 2, (6, 32000)).astype(np.float32)
    _, _, p = orc.sample_batch(x, 1.0, 0.5, np.zeros(6, np.uint64), probs_out=True)
    fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    for r in range(6):
        row = p[r].copy()
        coin = float(rng.random())
        assert L.sample_argmax(fp(row), 32000) == orc.argmax(row)
        assert L.sample_mult(fp(row), 32000, coin) == orc.mult(row, np.float32(coin))
        for tp in (0.9, 0.5, 1.0, 0.0):
            assert L.sample_topp(fp(row), 32000, tp, None, coin) == orc.topp(row, tp, np.float32(coin)), tp
        assert np.array_equal(row, p[r])  # these entry points do not write the buffer


EDGE = [
    ("nan_row_mult", lambda r: np.tile(np.array([1.0, np.nan, 2.0, 0.5] * 8, np.float32), (r, 1)), 1.0, 1.0),
    ("neg_inf_row_mult", lambda r: np.full((r, 33), -np.inf, np.float32), 0.9, 1.0),
    ("flat_topp", lambda r: np.zeros((r, 32000), np.float32), 1.0, 0.9),
    ("flat_topp_near_one", lambda r: np.random.default_rng(6).normal(0, 0.1, (r, 32000)).astype(np.float32), 1.0, 0.9999),
    ("topp_tiny", lambda r: np.random.default_rng(5).normal(0, 1, (r, 513)).astype(np.float32), 1.3, 0.01),
    ("odd_vocab", lambda r: np.random.default_rng(12).normal(0, 2, (r, 31999)).astype(np.float32), 0.9, 0.9),
    ("tiny_vocab", lambda r: np.random.default_rng(10).normal(0, 1, (r, 3)).astype(np.float32), 1.0, 0.5),
    ("max_vocab", lambda r: np.random.default_rng(13).normal(0, 2, (r, 32768)).astype(np.float32), 0.7, 0.95),
    ("negative_temperature", lambda r: np.random.default_rng(9).normal(0, 1, (r, 301)).astype(np.float32), -0.5, 0.9),
    # full vocabulary: the streaming kernel's own path for T < 0 (the row's
    # minimum plays the maximum's part once divided by T)
    ("negative_temperature_wide", lambda r: np.random.default_rng(25).normal(0, 2, (r, 32000)).astype(np.float32),
     -0.7, 0.9),
    ("negative_temperature_mult", lambda r: np.random.default_rng(26).normal(0, 1.5, (r, 32000)).astype(np.float32),
     -0.9, 1.0),
    ("huge_logits", lambda r: np.random.default_rng(14).normal(0, 60, (r, 4000)).astype(np.float32), 1.0, 0.9),
]


EDGE_CASES_FAST = EDGE + [
    ("nan_in_topp_row", lambda r: np.tile(np.array([1.0, np.nan] + [0.5] * 30, np.float32), (r, 1)), 1.0, 0.9),
    ("one_hot", lambda r: np.where(np.arange(32000) == 777, 30.0, 0.0).astype(np.float32)[None, :].repeat(r, 0), 1.0, 0.9),
    ("nan_first_wide", lambda r: _with(np.random.default_rng(16).normal(0, 2, (r, 32000)), [0], np.nan), 0.8, 0.9),
    ("nan_middle_wide", lambda r: _with(np.random.default_rng(17).normal(0, 2, (r, 32000)), [20001], np.nan), 0.8, 0.9),
    ("wide_spread", lambda r: np.random.default_rng(18).normal(0, 30, (r, 32000)).astype(np.float32), 0.7, 0.9),
    ("tiny_logits", lambda r: np.random.default_rng(19).normal(0, 1e-30, (r, 32000)).astype(np.float32), 1.0, 0.9),
    ("some_tiny_logits", lambda r: _with(np.random.default_rng(20).normal(0, 2, (r, 32000)), list(range(0, 32000, 97)),
                                         1e-30), 0.7, 0.9),
    # the eight largest logits of each row copied to two more places: short
    # equal-p runs among the top candidates, ordered by index like glibc qsort
    ("tied_candidates", lambda r: _tied_top(np.random.default_rng(21).normal(0, 2, (r, 32000)), 8, 2), 0.8, 0.9),
    # temperatures outside [2^-10, 2^10]: rows the streaming kernel defers
    ("tiny_temperature", lambda r: np.random.default_rng(22).normal(0, 1, (r, 32000)).astype(np.float32), 1e-4, 0.9),
    ("huge_temperature", lambda r: np.random.default_rng(23).normal(0, 2, (r, 32000)).astype(np.float32), 3000.0, 0.9),
]


def _tied_top(x, top, copies):
    x = x.astype(np.float32)
    rng = np.random.default_rng(24)
    for row in x:
        for j in np.argsort(row)[-top:]:
            row[rng.choice(len(row), copies, replace=False)] = row[j]
    return x


def _with(x, cols, value):
    x = x.astype(np.float32)
    x[:, cols] = value
    return x


@pytest.mark.parametrize("name,make,temp,topp", EDGE)
def test_edge_cases(pkg, orc, name, make, temp, topp):
    x = make(24)
    seeds = np.arange(24, dtype=np.uint64) * 11 + 5
    out = gpu_sample(pkg, x, temp, topp, seeds=seeds, want_probs=True)
    ref_ids, ref_st, ref_p = orc.sample_batch(x, temp, topp, seeds, probs_out=True)
    assert np.array_equal(out["states"], ref_st)
    finite = np.isfinite(ref_p)
    assert np.array_equal(np.isnan(out["probs"]), np.isnan(ref_p))
    rel, _ = prob_rel_err(np.where(finite, out["probs"], 0), np.where(finite, ref_p, 0))
    assert rel <= PROB_RTOL
    nan_rows = np.isnan(ref_p).any(axis=1)
    if nan_rows.any() and not (topp <= 0 or topp >= 1):
        # the reference reads probindex[-1] here (no candidates); flagged, id 0
        assert (out["flags"][nan_rows] & pkg.ROW_NO_CANDIDATE).all()
        keep = ~nan_rows
    else:
        keep = np.ones(len(x), bool)
    check_e2e(orc, out["ids"][keep], ref_ids[keep], ref_p[keep], seeds[keep], np.full(keep.sum(), topp))


def test_large_nucleus_takes_global_path(pkg, orc):
    x = np.random.default_rng(15).normal(0, 0.05, (8, 32000)).astype(np.float32)
    seeds = np.arange(8, dtype=np.uint64) + 100
    out = gpu_sample(pkg, x, 1.0, 0.95, seeds=seeds, want_probs=True)
    assert (out["flags"] & pkg.ROW_SLOW_PATH).all()
    ref_ids, _, ref_p = orc.sample_batch(x, 1.0, 0.95, seeds, probs_out=True)
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, np.full(8, 0.95))


def test_unaligned_row_stride(pkg, orc):
    """ld not a multiple of 4: rows are staged with plain loads."""
    x = np.random.default_rng(16).normal(0, 2, (20, 1001)).astype(np.float32)
    seeds = np.arange(20, dtype=np.uint64)
    out = gpu_sample(pkg, x, 0.9, 0.9, seeds=seeds, ld=1003)
    ref_ids, ref_st, ref_p = orc.sample_batch(x, 0.9, 0.9, seeds, probs_out=True)
    assert np.array_equal(out["states"], ref_st)
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, np.full(20, 0.9))


@pytest.mark.parametrize("want_probs", [False, True])
def test_partial_last_chunk_and_16_byte_rows(pkg, orc, want_probs):
    """The streaming kernel with V = 32004 (its last chunk of 32 holds 4
    values) and a row stride of 32012 floats (rows 16- but not 32-byte
    aligned, so chunks load as 16-byte vectors)."""
    x = np.random.default_rng(27).normal(0, 2, (24, 32004)).astype(np.float32)
    seeds = np.arange(24, dtype=np.uint64) * 3 + 1
    topps = np.where(np.arange(24) % 3 == 0, 1.0, 0.9).astype(np.float32)
    out = gpu_sample(pkg, x, 0.8, 0.9, seeds=seeds, topp_rows=topps, ld=32012, want_probs=want_probs)
    ref_ids, ref_st, ref_p = orc.sample_batch(x, 0.8, 0.9, seeds, topp_rows=topps, probs_out=True)
    assert np.array_equal(out["states"], ref_st)
    assert not (out["flags"] & pkg.ROW_SLOW_PATH).any()
    if want_probs:
        rel, zero_ok = prob_rel_err(out["probs"], ref_p)
        assert rel <= PROB_RTOL and zero_ok, rel
    check_e2e(orc, out["ids"], ref_ids, ref_p, seeds, topps)


def test_host_buffer_entry_point(pkg, orc):
    w = pkg.workloads.topp(rows=700)
    st = pkg.workloads.row_seeds(700)
    ids = pkg.sample_batched_host(w["logits"], 0.7, 0.9, st, topp_rows_np=w["topp_rows"])
    ref_ids, ref_st, ref_p = orc.sample_batch(w["logits"], 0.7, 0.9, pkg.workloads.row_seeds(700),
                                              topp_rows=w["topp_rows"], probs_out=True)
    assert np.array_equal(st, ref_st)
    check_e2e(orc, ids, ref_ids, ref_p, pkg.workloads.row_seeds(700), w["topp_rows"])


def test_repeatable(pkg):
    w = pkg.workloads.topp(rows=300)
    seeds = pkg.workloads.row_seeds(300)
    a = gpu_sample(pkg, w["logits"], 0.7, 0.9, seeds=seeds, topp_rows=w["topp_rows"])
    b = gpu_sample(pkg, w["logits"], 0.7, 0.9, seeds=seeds, topp_rows=w["topp_rows"])
    assert np.array_equal(a["ids"], b["ids"]) and np.array_equal(a["states"], b["states"])


@pytest.mark.parametrize("name,make,temp,topp", EDGE_CASES_FAST)
def test_edge_cases_pipelined(pkg, orc, name, make, temp, topp):
    x = make(24)
    seeds = np.arange(24, dtype=np.uint64) * 11 + 5
    out = gpu_sample(pkg, x, temp, topp, seeds=seeds)
    ref_ids, ref_st, ref_p = orc.sample_batch(x, temp, topp, seeds, probs_out=True)
    assert np.array_equal(out["states"], ref_st)
    nan_rows = np.isnan(ref_p).any(axis=1)
    keep = ~nan_rows if (nan_rows.any() and 0 < topp < 1) else np.ones(len(x), bool)
    if nan_rows.any() and 0 < topp < 1:
        assert (out["flags"][nan_rows] & pkg.ROW_NO_CANDIDATE).all()
    check_e2e(orc, out["ids"][keep], ref_ids[keep], ref_p[keep], seeds[keep], np.full(keep.sum(), topp))


def test_concurrent_samplers_on_threads(pkg):
    """Distinct Samplers used from different threads are independent (as in
    the reference): concurrent sample() calls give the ids a sequential run
    gives."""
    from concurrent.futures import ThreadPoolExecutor
    rows = np.random.default_rng(33).normal(0, 2, (4, 40, 32000)).astype(np.float32)

    def run(t):
        s = pkg.build_sampler(32000, 0.9, 0.9, 100 + t)
        ids = [pkg.sample(s, rows[t, r].copy()) for r in range(rows.shape[1])]
        pkg.free_sampler(s)
        return ids

    want = [run(t) for t in range(4)]
    with ThreadPoolExecutor(4) as ex:
        got = list(ex.map(run, range(4)))
    assert got == want


# ---------------------------------------------------------------------------
# sample_debug (llama2_cublas.cu:5067-5111) and do_sample
# (llama2_cublas_fp16.cu:1178-1189): the mode flags of the batched call and
# the two single-row entry points, against tests/golden/modes.json (the
# reference's own functions) and the oracle
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("want_probs", [True, False])
def test_mode_rules_batched(pkg, orc, golden, want_probs):
    w = pkg.workloads.debug_rows()
    x = w["logits"]
    B = x.shape[0]
    seeds = pkg.workloads.row_seeds(B)
    nan_rows = np.isnan(x).any(axis=1)
    for case in golden["modes"]["cases"]:
        mode, temp, topp = case["mode"], case["temperature"], case["topp"]
        out = gpu_sample(pkg, x, temp, topp, seeds=seeds, want_probs=want_probs, mode=mode)
        assert out["states"].tolist() == case["states_after"], case["entry"]
        ref_ids, _, ref_p = orc.sample_batch(x, temp, topp, seeds, probs_out=True, mode=mode)
        gids = np.array(case["ids"])
        greedy = np.float32(temp) < np.float32(1e-6)
        if mode & pkg.SAMPLER_FLAG_NAN_TOKEN1:
            assert (out["ids"][nan_rows] == 1).all() and (out["flags"][nan_rows] & pkg.ROW_NAN).all()
            if want_probs:  # the buffer keeps the logits
                assert np.array_equal(out["probs"][nan_rows].view(np.uint32), x[nan_rows].view(np.uint32))
            keep = ~nan_rows
        else:
            keep = np.ones(B, bool) if greedy else ~nan_rows  # NaN rows: undefined id in the reference
        if greedy:
            assert np.array_equal(out["ids"][keep], gids[keep])  # argmax: bit-exact
        else:
            check_e2e(orc, out["ids"][keep], gids[keep], ref_p[keep], seeds[keep], np.full(keep.sum(), topp))
            if want_probs:
                rel, _ = prob_rel_err(out["probs"][keep], ref_p[keep])
                assert rel <= PROB_RTOL


def test_mode_rules_greedy_threshold_per_row(pkg, golden):
    """Per-row temperatures on both sides of 1e-6f in one batch: greedy rows
    under GREEDY_BELOW_1E6 draw nothing; without the flag only T == 0 is."""
    w = pkg.workloads.debug_rows()
    x = w["logits"][~np.isnan(w["logits"]).any(axis=1)][:32]
    temps = np.array([5e-7, 0.8, -0.5, 1e-6, 0.0, 9.9e-7, 0.7, 2e-6] * 4, np.float32)
    seeds = np.arange(32, dtype=np.uint64) + 9
    out = gpu_sample(pkg, x, 0.8, 0.9, seeds=seeds, temp_rows=temps, mode=pkg.MODE_DO_SAMPLE)
    greedy = temps < np.float32(1e-6)
    assert np.array_equal(out["states"][greedy], seeds[greedy])
    assert (out["states"][~greedy] != seeds[~greedy]).all()
    assert out["ids"][greedy].tolist() == [int(np.argmax(r)) for r in x[greedy]]
    plain = gpu_sample(pkg, x, 0.8, 0.9, seeds=seeds, temp_rows=temps)
    assert np.array_equal(plain["states"] == seeds, temps == 0.0)


@pytest.mark.parametrize("entry,mode", [("sample_debug", 6), ("do_sample", 2)])
def test_mode_rules_single_row_entry_points(pkg, orc, entry, mode):
    """llama2_cublas.cu:5905 / llama2_cublas_fp16.cu:1268 call sites: one
    Sampler advancing over rows, the buffer written back as the reference
    leaves it."""
    w = pkg.workloads.debug_rows(rows=22)
    x = w["logits"]
    for temp in (0.8, 5e-7, -0.5):
        s = pkg.build_sampler(x.shape[1], temp, 0.9, 42)
        st = np.array([42], np.uint64)
        for r in range(x.shape[0]):
            row = x[r].copy()
            got = pkg.sample(s, row, entry=entry)
            ref_ids, ref_st, ref_p = orc.sample_batch(x[r:r + 1], temp, 0.9, st, probs_out=True, mode=mode)
            assert s.rng_state == int(ref_st[0]), (entry, temp, r)
            nan_row = bool(np.isnan(x[r]).any())
            if nan_row and mode & 4:
                assert got == 1 and np.array_equal(row.view(np.uint32), x[r].view(np.uint32))
            elif np.float32(temp) < np.float32(1e-6):
                assert got == int(ref_ids[0]) and np.array_equal(row.view(np.uint32), x[r].view(np.uint32))
            elif not nan_row:
                rel, _ = prob_rel_err(row[None, :], ref_p)
                assert rel <= PROB_RTOL
                if got != int(ref_ids[0]):
                    coin, _ = orc.coin(int(st[0]))
                    assert orc.boundary_distance(ref_p[0], 0.9, coin) <= BOUNDARY
            st = ref_st
        pkg.free_sampler(s)
