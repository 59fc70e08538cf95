"""CPU: the oracle restatement against the reference's own sampler and the
golden ids that sampler produced (tests/golden/gen_golden.py)."""
import hashlib

import numpy as np
import pytest


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def test_inputs_match_golden(pkg, golden):
    wl = pkg.workloads
    assert digest(wl.single_row()["logits"]) == golden["single_row"]["input_sha"]
    assert digest(wl.argmax()["logits"]) == golden["argmax"]["input_sha"]
    assert digest(wl.mult()["logits"]) == golden["mult"]["input_sha"]


def test_oracle_single_row_sequence(pkg, orc, golden):
    w = pkg.workloads.single_row()
    ids = orc.sample_sequence(w["logits"], w["temperature"], w["topp"], w["seed"])
    assert ids.tolist() == golden["single_row"]["ids"]


def test_oracle_argmax_batch(pkg, orc, golden):
    w = pkg.workloads.argmax()
    ids, _ = orc.sample_batch(w["logits"], 0.0, 0.9, pkg.workloads.row_seeds(256))
    assert ids.tolist() == golden["argmax"]["ids"]


def test_oracle_mult_batch(pkg, orc, golden):
    w = pkg.workloads.mult()
    ids, st = orc.sample_batch(w["logits"], w["temperature"], w["topp"], pkg.workloads.row_seeds(1024))
    assert ids.tolist() == golden["mult"]["ids"]
    assert [int(x) for x in st[:8]] == golden["mult"]["states_after"]


def test_oracle_topp_batch(pkg, orc, golden):
    w = pkg.workloads.topp()
    assert digest(w["logits"]) == golden["topp"]["input_sha"]
    ids, _ = orc.sample_batch(w["logits"], w["temperature"], w["topp"], pkg.workloads.row_seeds(4096),
                              topp_rows=w["topp_rows"])
    assert ids.tolist() == golden["topp"]["ids"]
    assert golden["topp"]["nucleus_min"] == 1 and golden["topp"]["nucleus_max"] > 1000


def test_oracle_probs_in(pkg, orc, golden):
    wl = pkg.workloads
    _, _, pm = orc.sample_batch(wl.mult(rows=256)["logits"], 0.8, 1.0, wl.row_seeds(256), probs_out=True)
    w = wl.topp(rows=256)
    _, _, pt = orc.sample_batch(w["logits"], 0.7, 0.9, wl.row_seeds(256), topp_rows=w["topp_rows"], probs_out=True)
    g = golden["probs_in"]
    assert digest(pm) == g["mult_probs_sha"] and digest(pt) == g["topp_probs_sha"]
    ids_m, _ = orc.sample_probs_batch(pm, 1.0, wl.row_seeds(256))
    ids_t, _ = orc.sample_probs_batch(pt, 0.9, wl.row_seeds(256), topp_rows=w["topp_rows"])
    assert ids_m.tolist() == g["mult_ids"] and ids_t.tolist() == g["topp_ids"]


EDGE_CASES = [
    # (name, rows builder, temperature, topp)
    ("ties_and_zero", lambda r: np.tile(np.array([0.0, -0.0, 3.0, 3.0, 1.0], np.float32), (r, 1)), 0.0, 0.9),
    ("nan_first", lambda r: np.tile(np.array([np.nan, 1.0, 2.0, 2.0], np.float32), (r, 1)), 0.0, 0.9),
    ("nan_later_mult", lambda r: np.tile(np.array([1.0, np.nan, 2.0, 0.5], np.float32), (r, 1)), 1.0, 1.0),
    ("all_neg_inf_mult", lambda r: np.full((r, 7), -np.inf, np.float32), 0.9, 1.0),
    ("flat_topp", lambda r: np.zeros((r, 1000), np.float32), 1.0, 0.9),
    ("topp_tiny", lambda r: np.random.default_rng(5).normal(0, 1, (r, 513)).astype(np.float32), 1.3, 0.01),
    ("topp_near_one", lambda r: np.random.default_rng(6).normal(0, 1, (r, 2000)).astype(np.float32), 0.5, 0.9999),
    ("topp_zero_mult", lambda r: np.random.default_rng(8).normal(0, 1, (r, 300)).astype(np.float32), 1.0, 0.0),
    ("negative_temperature", lambda r: np.random.default_rng(9).normal(0, 1, (r, 301)).astype(np.float32), -0.5, 0.9),
    ("vocab_two", lambda r: np.random.default_rng(10).normal(0, 1, (r, 2)).astype(np.float32), 1.0, 0.5),
]


@pytest.mark.parametrize("name,make,temp,topp", EDGE_CASES)
def test_oracle_matches_reference_edge_cases(ref, orc, name, make, temp, topp):
    x = make(16)
    seeds = np.arange(16, dtype=np.uint64) + 7
    a, sa, pa = ref.sample_batch(x, temp, topp, seeds, probs_out=True)
    b, sb, pb = orc.sample_batch(x, temp, topp, seeds, probs_out=True)
    assert np.array_equal(a, b) and np.array_equal(sa, sb)
    assert np.array_equal(pa.view(np.uint32), pb.view(np.uint32))


def test_oracle_matches_reference_random(ref, orc):
    rng = np.random.default_rng(11)
    for V, sigma, temp, topp in [(32000, 2.0, 1.0, 0.9), (4099, 4.0, 0.6, 0.95), (777, 0.5, 1.7, 0.5)]:
        x = rng.normal(0, sigma, (32, V)).astype(np.float32)
        seeds = np.arange(32, dtype=np.uint64) * 3 + 1
        a, sa = ref.sample_batch(x, temp, topp, seeds)
        b, sb = orc.sample_batch(x, temp, topp, seeds)
        assert np.array_equal(a, b) and np.array_equal(sa, sb)


def test_reference_baseline_threads(ref):
    assert ref.num_threads() >= 1


def test_oracle_sample_debug_and_do_sample(pkg, orc, golden):
    """The restated sample_debug / do_sample rules against the reference's own
    functions (tests/golden/modes.json, written by the reference's code cut out
    of llama2_cublas.cu and llama2_cublas_fp16.cu).  Rows whose top-p walk
    finds no candidate (a NaN row without the NaN guard) read probindex[-1] in
    the reference, an undefined id; there the oracle returns -1 and only the
    state and the buffer are compared."""
    w = pkg.workloads.debug_rows()
    g = golden["modes"]
    assert digest(w["logits"]) == g["input_sha"]
    seeds = pkg.workloads.row_seeds(w["logits"].shape[0])
    for case in g["cases"]:
        ids, st, pr = orc.sample_batch(w["logits"], case["temperature"], case["topp"], seeds, probs_out=True,
                                       mode=case["mode"])
        defined = ids >= 0
        assert np.array_equal(ids[defined], np.array(case["ids"])[defined]), case["entry"]
        assert [int(x) for x in st] == case["states_after"]
        assert digest(pr) == case["probs_sha"]
        if case["mode"] & 4:  # NaN rows: token 1, no draw
            nan_rows = np.isnan(w["logits"]).any(axis=1)
            assert (ids[nan_rows] == 1).all() and np.array_equal(st[nan_rows], seeds[nan_rows])
