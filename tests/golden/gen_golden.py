"""Generates the golden token ids in tests/golden/ by running the REFERENCE's
own sampler (oracle/_ref/libref_sampler.so, compiled from the reference's
llama2_cublas_fp16.c by oracle/Makefile) on the seeded synthetic workloads.

Run in a tree where the reference sources exist:
    python tests/golden/gen_golden.py
Outputs (small JSON files, committed):
    single_row.json  256 ids of one sampler (seed 42) advancing over 256 rows
    argmax.json      256 greedy ids (with planted ties)
    mult.json        1024 sample_mult ids, per-row seeds 42+row
    topp.json        4096 sample_topp ids, per-row seeds 42+row, plus nucleus stats
    probs_in.json    sample_mult / sample_topp ids given the reference's own
                     probabilities (first 256 rows of mult and topp)
    modes.json       sample_debug / do_sample ids and states on rows with NaNs,
                     over temperatures around the 1e-6 greedy threshold
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from __graft_entry__ import load_package  # noqa: E402


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def nucleus_sizes(probs, topps):
    out = []
    for p, tp in zip(probs, topps):
        s = np.sort(p[p >= (1.0 - tp) / (p.shape[0] - 1)])[::-1]
        c = np.cumsum(s, dtype=np.float64)
        out.append(int(np.searchsorted(c, tp, side="right") + 1))
    return out


def main():
    oracle.build(with_ref=True)
    ref = oracle.ref_sampler()
    wl = load_package().workloads

    w = wl.single_row()
    ids = ref.sample_sequence(w["logits"], w["temperature"], w["topp"], w["seed"])
    json.dump(dict(workload="single_row", input_sha=digest(w["logits"]), ids=ids.tolist()),
              open(os.path.join(HERE, "single_row.json"), "w"))

    w = wl.argmax()
    ids, _ = ref.sample_batch(w["logits"], 0.0, w["topp"], wl.row_seeds(256))
    json.dump(dict(workload="argmax", input_sha=digest(w["logits"]), ids=ids.tolist()),
              open(os.path.join(HERE, "argmax.json"), "w"))

    w = wl.mult()
    ids, st, probs_m = ref.sample_batch(w["logits"], w["temperature"], w["topp"], wl.row_seeds(1024), probs_out=True)
    json.dump(dict(workload="mult", input_sha=digest(w["logits"]), ids=ids.tolist(),
                   states_after=[int(x) for x in st[:8]]),
              open(os.path.join(HERE, "mult.json"), "w"))

    w = wl.topp()
    ids, st, probs_t = ref.sample_batch(w["logits"], w["temperature"], w["topp"], wl.row_seeds(4096),
                                        topp_rows=w["topp_rows"], probs_out=True)
    ns = nucleus_sizes(probs_t, w["topp_rows"])
    json.dump(dict(workload="topp", input_sha=digest(w["logits"]), ids=ids.tolist(),
                   nucleus_min=min(ns), nucleus_max=max(ns), nucleus_mean=float(np.mean(ns))),
              open(os.path.join(HERE, "topp.json"), "w"))
    print("topp nucleus sizes: min %d max %d mean %.1f" % (min(ns), max(ns), np.mean(ns)))

    # probabilities-in: the reference's own probabilities, coins from 42+row
    pm, pt = probs_m[:256], probs_t[:256]
    ids_m, _ = ref.sample_probs_batch(pm, 1.0, wl.row_seeds(256))
    ids_t, _ = ref.sample_probs_batch(pt, 0.9, wl.row_seeds(256), topp_rows=w["topp_rows"][:256])
    json.dump(dict(mult_probs_sha=digest(pm), topp_probs_sha=digest(pt), mult_ids=ids_m.tolist(),
                   topp_ids=ids_t.tolist()),
              open(os.path.join(HERE, "probs_in.json"), "w"))
    # sample_debug (llama2_cublas.cu:5067-5111) and do_sample
    # (llama2_cublas_fp16.cu:1178-1189) of the reference's CUDA translation
    # units, built from their sources into oracle/_ref (oracle/Makefile)
    w = wl.debug_rows()
    seeds = wl.row_seeds(w["logits"].shape[0])
    cases = []
    for mode, name in ((6, "sample_debug"), (2, "do_sample")):
        for temp in w["temperatures"]:
            for tp in w["topps"]:
                ids, st, pr = ref.sample_batch(w["logits"], temp, tp, seeds, probs_out=True, mode=mode)
                cases.append(dict(entry=name, mode=mode, temperature=temp, topp=tp, ids=ids.tolist(),
                                  states_after=[int(x) for x in st], probs_sha=digest(pr)))
    json.dump(dict(workload="debug_rows", input_sha=digest(w["logits"]), cases=cases),
              open(os.path.join(HERE, "modes.json"), "w"))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
