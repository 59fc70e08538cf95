"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checker libraries.

liboracle.so          the CPU restatement of the llama2.c sampler
_ref/libref_sampler.so the reference's own sampler built from its sources

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline leg use this
module; the product library never loads it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_sampler.so")


def build(with_ref=True):
    """Builds liboracle.so and, when the reference sources are reachable
    (oracle/Makefile's REF_DIR, or the REFERENCE_DIR environment variable),
    _ref/libref_sampler.so.  Where they are absent (the GPU box) the prebuilt
    _ref library is used as it is."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if with_ref:
        r = subprocess.run(["make", "-s", "-C", HERE, "ref"], stdout=subprocess.DEVNULL,
                           stderr=subprocess.DEVNULL)
        if r.returncode != 0 and not os.path.exists(REF_SO):
            return False
    return True


_P = ctypes.c_void_p


def _fp(a):
    return a.ctypes.data_as(_P)


class _Lib:
    def __init__(self, path, prefix):
        self.L = ctypes.CDLL(path)
        self.prefix = prefix
        L = self.L
        f = getattr(L, prefix + "sample_batch")
        f.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_float, _P, _P,
                      _P, _P, ctypes.c_int]
        f.restype = ctypes.c_int
        f = getattr(L, prefix + "sample_mode_batch")
        f.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_float, _P, _P,
                      _P, _P, ctypes.c_int, ctypes.c_int]
        f.restype = ctypes.c_int
        f = getattr(L, prefix + "sample_probs_batch")
        f.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, _P, _P, _P, ctypes.c_int]
        f.restype = ctypes.c_int
        f = getattr(L, prefix + "sample_sequence")
        f.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_ulonglong, _P]
        f.restype = ctypes.c_int

    def sample_batch(self, logits, temperature, topp, states, topp_rows=None, probs_out=False, nthreads=0,
                     mode=0):
        """sample() per row; mode 6 = sample_debug, mode 2 = do_sample (the
        per-row calls of the reference's CUDA translation units)."""
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        B, V = logits.shape
        ids = np.empty(B, dtype=np.int32)
        st = np.array(states, dtype=np.uint64, copy=True)
        tr = None if topp_rows is None else np.ascontiguousarray(topp_rows, dtype=np.float32)
        pr = np.empty_like(logits) if probs_out else None
        args = (_fp(logits), B, V, V, temperature, topp, None if tr is None else _fp(tr), _fp(st), _fp(ids),
                None if pr is None else _fp(pr), nthreads)
        if mode:
            rc = getattr(self.L, self.prefix + "sample_mode_batch")(*args, mode)
            if rc != 0:
                raise ValueError(f"mode {mode} not available in {self.prefix}sample_mode_batch")
        else:
            getattr(self.L, self.prefix + "sample_batch")(*args)
        return (ids, st, pr) if probs_out else (ids, st)

    def sample_probs_batch(self, probs, topp, states, topp_rows=None, nthreads=0):
        probs = np.ascontiguousarray(probs, dtype=np.float32)
        B, V = probs.shape
        ids = np.empty(B, dtype=np.int32)
        st = np.array(states, dtype=np.uint64, copy=True)
        tr = None if topp_rows is None else np.ascontiguousarray(topp_rows, dtype=np.float32)
        getattr(self.L, self.prefix + "sample_probs_batch")(
            _fp(probs), B, V, V, topp, None if tr is None else _fp(tr), _fp(st), _fp(ids), nthreads)
        return ids, st

    def sample_sequence(self, logits, temperature, topp, seed):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        S, V = logits.shape
        ids = np.empty(S, dtype=np.int32)
        getattr(self.L, self.prefix + "sample_sequence")(_fp(logits), S, V, temperature, topp, seed, _fp(ids))
        return ids


class Oracle(_Lib):
    def __init__(self):
        super().__init__(ORACLE_SO, "oracle_")
        L = self.L
        L.oracle_boundary_distance.argtypes = [_P, ctypes.c_int, ctypes.c_float, ctypes.c_float]
        L.oracle_boundary_distance.restype = ctypes.c_double
        L.oracle_random_f32.argtypes = [ctypes.POINTER(ctypes.c_ulonglong)]
        L.oracle_random_f32.restype = ctypes.c_float
        L.oracle_softmax_sum.argtypes = [_P, ctypes.c_int, ctypes.c_float]
        L.oracle_softmax_sum.restype = ctypes.c_float
        L.oracle_argmax.argtypes = [_P, ctypes.c_int]
        L.oracle_argmax.restype = ctypes.c_int
        L.oracle_mult.argtypes = [_P, ctypes.c_int, ctypes.c_float]
        L.oracle_mult.restype = ctypes.c_int
        L.oracle_topp.argtypes = [_P, ctypes.c_int, ctypes.c_float, _P, ctypes.c_float]
        L.oracle_topp.restype = ctypes.c_int

    def argmax(self, p):
        p = np.ascontiguousarray(p, dtype=np.float32)
        return self.L.oracle_argmax(_fp(p), p.shape[0])

    def mult(self, p, coin):
        p = np.ascontiguousarray(p, dtype=np.float32)
        return self.L.oracle_mult(_fp(p), p.shape[0], coin)

    def topp(self, p, topp, coin):
        p = np.ascontiguousarray(p, dtype=np.float32)
        scratch = np.empty(2 * p.shape[0], dtype=np.int32)
        return self.L.oracle_topp(_fp(p), p.shape[0], topp, _fp(scratch), coin)

    def boundary_distance(self, probs_row, topp, coin):
        p = np.ascontiguousarray(probs_row, dtype=np.float32)
        return self.L.oracle_boundary_distance(_fp(p), p.shape[0], topp, coin)

    def coin(self, state):
        s = ctypes.c_ulonglong(int(state))
        c = self.L.oracle_random_f32(ctypes.byref(s))
        return c, s.value


class RefSampler(_Lib):
    def __init__(self):
        super().__init__(REF_SO, "ref_")
        self.L.ref_num_threads.restype = ctypes.c_int

    def num_threads(self):
        return self.L.ref_num_threads()


def oracle():
    if not os.path.exists(ORACLE_SO):
        build(with_ref=False)
    return Oracle()


def ref_available():
    return os.path.exists(REF_SO)


def ref_sampler():
    return RefSampler()
