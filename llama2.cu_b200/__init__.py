"""Python bindings of libb200_sampler.so (the C-ABI in include/b200_sampler.h).

The package directory is named ``llama2.cu_b200``; load it with
``load_package()`` from ``__graft_entry__`` / tests (the dot in the name keeps
it out of the normal import path).  Everything here is a thin ctypes layer:
the sampling itself runs in the library's sm_100a kernels, and every call
fails loudly (``SamplerError``) when the library or a GPU is missing.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200_sampler.so")

SAMPLER_FLAG_PROBS_IN = 1
SAMPLER_FLAG_GREEDY_BELOW_1E6 = 2
SAMPLER_FLAG_NAN_TOKEN1 = 4
MODE_DO_SAMPLE = SAMPLER_FLAG_GREEDY_BELOW_1E6
MODE_SAMPLE_DEBUG = SAMPLER_FLAG_GREEDY_BELOW_1E6 | SAMPLER_FLAG_NAN_TOKEN1
ROW_NAN, ROW_NO_CANDIDATE, ROW_SLOW_PATH, ROW_SERIAL, ROW_TIMEOUT = 1, 2, 4, 8, 16
MAX_VOCAB = 32768

# Every symbol the header declares (the CPU tests check the library exports them).
EXPORTED_SYMBOLS = [
    "build_sampler", "free_sampler", "random_u32", "random_f32", "sample_argmax", "sample_mult",
    "sample_topp", "sample", "sample_debug", "do_sample", "sampler_workspace_bytes", "sampler_batched", "sampler_batched_host",
    "sampler_seed_states", "sampler_last_launch_count", "sampler_last_error", "sampler_shard_rows",
    "sampler_nccl_get_unique_id", "sampler_nccl_comm_init", "sampler_nccl_allgather_ids",
    "sampler_nccl_comm_destroy", "sampler_batched_noalloc", "classifier_sample_fused",
    "classifier_logits", "rmsnorm_bf16", "classifier_rmsnorm_sample_fused", "sampler_gather_rows",
    "sampler_selftest_wait_timeout",
]


class SamplerError(RuntimeError):
    pass


class ProbIndex(ctypes.Structure):
    _fields_ = [("prob", ctypes.c_float), ("index", ctypes.c_int)]


class Sampler(ctypes.Structure):
    """Same layout as llama2.c's Sampler (llama2.c:973-979)."""
    _fields_ = [("vocab_size", ctypes.c_int), ("probindex", ctypes.POINTER(ProbIndex)),
                ("temperature", ctypes.c_float), ("topp", ctypes.c_float),
                ("rng_state", ctypes.c_ulonglong)]


class SamplerBatchConfig(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int), ("temperature", ctypes.c_float),
                ("topp", ctypes.c_float), ("flags", ctypes.c_int)]


_lib = None


def library_path():
    return LIB_PATH


def lib():
    """Loads the library (RTLD_LOCAL) and declares the prototypes."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise SamplerError(f"{LIB_PATH} is missing: build it with llama2.cu_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    P, c_int, c_float, c_ull, c_size = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_ulonglong, ctypes.c_size_t
    fp = ctypes.POINTER(c_float)
    L.build_sampler.argtypes = [ctypes.POINTER(Sampler), c_int, c_float, c_float, c_ull]
    L.build_sampler.restype = None
    L.free_sampler.argtypes = [ctypes.POINTER(Sampler)]
    L.free_sampler.restype = None
    L.random_u32.argtypes = [ctypes.POINTER(c_ull)]
    L.random_u32.restype = ctypes.c_uint
    L.random_f32.argtypes = [ctypes.POINTER(c_ull)]
    L.random_f32.restype = c_float
    L.sample_argmax.argtypes = [fp, c_int]
    L.sample_argmax.restype = c_int
    L.sample_mult.argtypes = [fp, c_int, c_float]
    L.sample_mult.restype = c_int
    L.sample_topp.argtypes = [fp, c_int, c_float, ctypes.POINTER(ProbIndex), c_float]
    L.sample_topp.restype = c_int
    L.sample.argtypes = [ctypes.POINTER(Sampler), fp]
    L.sample.restype = c_int
    L.sample_debug.argtypes = [ctypes.POINTER(Sampler), fp]
    L.sample_debug.restype = c_int
    L.do_sample.argtypes = [ctypes.POINTER(Sampler), fp]
    L.do_sample.restype = c_int
    L.sampler_workspace_bytes.argtypes = [c_int, c_int]
    L.sampler_workspace_bytes.restype = c_size
    L.sampler_batched.argtypes = [ctypes.POINTER(SamplerBatchConfig), P, c_int, ctypes.c_longlong, P, P, P,
                                  P, P, P, P, P, c_size, P]
    L.sampler_batched.restype = c_int
    L.sampler_batched_host.argtypes = [ctypes.POINTER(SamplerBatchConfig), P, c_int, ctypes.c_longlong, P, P, P]
    L.sampler_batched_host.restype = c_int
    L.sampler_seed_states.argtypes = [P, c_int, c_ull, ctypes.c_longlong, P]
    L.sampler_seed_states.restype = c_int
    L.sampler_last_launch_count.argtypes = []
    L.sampler_last_launch_count.restype = c_int
    L.sampler_last_error.argtypes = []
    L.sampler_last_error.restype = ctypes.c_char_p
    L.sampler_shard_rows.argtypes = [c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]
    L.sampler_shard_rows.restype = c_int
    L.sampler_nccl_get_unique_id.argtypes = [P]
    L.sampler_nccl_get_unique_id.restype = c_int
    L.sampler_nccl_comm_init.argtypes = [ctypes.POINTER(P), c_int, P, c_int]
    L.sampler_nccl_comm_init.restype = c_int
    L.sampler_nccl_allgather_ids.argtypes = [P, P, c_int, P, P]
    L.sampler_nccl_allgather_ids.restype = c_int
    L.sampler_nccl_comm_destroy.argtypes = [P]
    L.sampler_nccl_comm_destroy.restype = c_int
    L.classifier_sample_fused.argtypes = [ctypes.POINTER(SamplerBatchConfig), P, P, c_int, c_int, P, P, P, P, P, P,
                                          P, P]
    L.classifier_sample_fused.restype = c_int
    L.classifier_logits.argtypes = [P, P, c_int, c_int, c_int, P, P]
    L.classifier_logits.restype = c_int
    L.rmsnorm_bf16.argtypes = [P, P, c_int, c_int, P, P]
    L.rmsnorm_bf16.restype = c_int
    L.classifier_rmsnorm_sample_fused.argtypes = [ctypes.POINTER(SamplerBatchConfig), P, P, P, c_int, c_int, P, P,
                                                  P, P, P, P, P, P]
    L.classifier_rmsnorm_sample_fused.restype = c_int
    L.sampler_gather_rows.argtypes = [P, c_int, c_int, P, c_int, P, P]
    L.sampler_gather_rows.restype = c_int
    L.sampler_selftest_wait_timeout.argtypes = [ctypes.c_uint, ctypes.POINTER(c_int)]
    L.sampler_selftest_wait_timeout.restype = c_int
    _lib = L
    return L


def _check(rc, what):
    if rc != 0:
        raise SamplerError(f"{what} failed ({rc}): {lib().sampler_last_error().decode()}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise SamplerError("device entry point given a CPU tensor")


def shard_rows(batch, world, rank):
    b, c = ctypes.c_int(), ctypes.c_int()
    _check(lib().sampler_shard_rows(batch, world, rank, ctypes.byref(b), ctypes.byref(c)), "sampler_shard_rows")
    return b.value, c.value


def seed_states(states, seed, row_offset=0, stream=None):
    """states: int64 CUDA tensor [B] (bit pattern of the uint64 states)."""
    _require_cuda(states)
    _check(lib().sampler_seed_states(_ptr(states), states.numel(), ctypes.c_ulonglong(seed), row_offset,
                                     _stream_ptr(stream)), "sampler_seed_states")


def _stream_ptr(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def sample_batched(logits, temperature, topp, rng_state=None, *, temperature_rows=None, topp_rows=None,
                   coins=None, out_ids=None, probs_out=None, row_flags=None, probs_in=False,
                   workspace=None, stream=None, mode=0):
    """Batched device sampling over the rows of a CUDA fp32 tensor [B, ld].

    rng_state: int64 CUDA tensor [B] advanced in place (uint64 bit patterns).
    mode: 0 (sample()'s rules), MODE_SAMPLE_DEBUG or MODE_DO_SAMPLE.
    Returns out_ids (int32 CUDA tensor [B]).  Asynchronous on `stream`.
    """
    import torch
    _require_cuda(logits, rng_state, temperature_rows, topp_rows, coins, probs_out, row_flags, workspace)
    if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
        raise SamplerError("logits must be a row-major float32 [B, ld] tensor")
    B, V = logits.shape
    if out_ids is None:
        out_ids = torch.empty(B, dtype=torch.int32, device=logits.device)
    cfg = SamplerBatchConfig(V, float(temperature), float(topp), (SAMPLER_FLAG_PROBS_IN if probs_in else 0) | mode)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = lib().sampler_batched(ctypes.byref(cfg), _ptr(logits), B, logits.stride(0), _ptr(temperature_rows),
                               _ptr(topp_rows), _ptr(coins), _ptr(rng_state), _ptr(out_ids), _ptr(probs_out),
                               _ptr(row_flags), _ptr(workspace), ws_bytes, _stream_ptr(stream))
    _check(rc, "sampler_batched")
    return out_ids


def classifier_sample_fused(hidden, wcls, temperature, topp, rng_state=None, *, temperature_rows=None,
                            topp_rows=None, coins=None, out_ids=None, logits_out=None, row_flags=None, stream=None):
    """Fused classifier + sampling: hidden bf16 CUDA [B, D], wcls bf16 CUDA
    [V, D]; logits = hidden . wcls^T (fp32, optionally returned in
    logits_out [B, V]) sampled per row as sample_batched() does.
    Returns out_ids (int32 CUDA tensor [B]).  Asynchronous on `stream`."""
    import torch
    _require_cuda(hidden, wcls, rng_state, temperature_rows, topp_rows, coins, logits_out, row_flags)
    for t in (hidden, wcls):
        if t.dtype != torch.bfloat16 or t.dim() != 2 or not t.is_contiguous():
            raise SamplerError("hidden and wcls must be contiguous bfloat16 matrices")
    B, D = hidden.shape
    V = wcls.shape[0]
    if wcls.shape[1] != D:
        raise SamplerError("hidden and wcls disagree on the model dimension")
    if logits_out is not None and (logits_out.dtype != torch.float32 or tuple(logits_out.shape) != (B, V)
                                   or not logits_out.is_contiguous()):
        raise SamplerError("logits_out must be a contiguous float32 [B, V] tensor")
    if out_ids is None:
        out_ids = torch.empty(B, dtype=torch.int32, device=hidden.device)
    cfg = SamplerBatchConfig(V, float(temperature), float(topp), 0)
    rc = lib().classifier_sample_fused(ctypes.byref(cfg), _ptr(hidden), _ptr(wcls), B, D, _ptr(temperature_rows),
                                       _ptr(topp_rows), _ptr(coins), _ptr(rng_state), _ptr(out_ids),
                                       _ptr(logits_out), _ptr(row_flags), _stream_ptr(stream))
    _check(rc, "classifier_sample_fused")
    return out_ids


def classifier_logits(hidden, wcls, logits_out=None, stream=None):
    """logits = hidden . wcls^T (bf16 in, fp32 out): tensor cores from three rows,
    a CUDA-core GEMV streaming wcls for one or two."""
    import torch
    _require_cuda(hidden, wcls, logits_out)
    B, D = hidden.shape
    V = wcls.shape[0]
    if logits_out is None:
        logits_out = torch.empty(B, V, dtype=torch.float32, device=hidden.device)
    rc = lib().classifier_logits(_ptr(hidden), _ptr(wcls), B, D, V, _ptr(logits_out), _stream_ptr(stream))
    _check(rc, "classifier_logits")
    return logits_out


def rmsnorm_bf16(x, norm_weight, out=None, stream=None):
    """bf16(norm_weight * x / rms(x)) per row of a float32 CUDA tensor [B, D]."""
    import torch
    _require_cuda(x, norm_weight, out)
    B, D = x.shape
    if out is None:
        out = torch.empty(B, D, dtype=torch.bfloat16, device=x.device)
    _check(lib().rmsnorm_bf16(_ptr(x), _ptr(norm_weight), B, D, _ptr(out), _stream_ptr(stream)), "rmsnorm_bf16")
    return out


def classifier_rmsnorm_sample_fused(x, norm_weight, wcls, temperature, topp, rng_state=None, *,
                                    temperature_rows=None, topp_rows=None, coins=None, out_ids=None,
                                    logits_out=None, row_flags=None, stream=None):
    """Decode step from fp32 hidden states [B, D]: final RMSNorm, classifier
    GEMM, sampling.  Returns out_ids (int32 CUDA tensor [B])."""
    import torch
    _require_cuda(x, norm_weight, wcls, rng_state, temperature_rows, topp_rows, coins, logits_out, row_flags)
    if x.dtype != torch.float32 or not x.is_contiguous() or wcls.dtype != torch.bfloat16:
        raise SamplerError("x must be contiguous float32 [B, D] and wcls bfloat16 [V, D]")
    B, D = x.shape
    V = wcls.shape[0]
    if out_ids is None:
        out_ids = torch.empty(B, dtype=torch.int32, device=x.device)
    cfg = SamplerBatchConfig(V, float(temperature), float(topp), 0)
    rc = lib().classifier_rmsnorm_sample_fused(ctypes.byref(cfg), _ptr(x), _ptr(norm_weight), _ptr(wcls), B, D,
                                               _ptr(temperature_rows), _ptr(topp_rows), _ptr(coins),
                                               _ptr(rng_state), _ptr(out_ids), _ptr(logits_out), _ptr(row_flags),
                                               _stream_ptr(stream))
    _check(rc, "classifier_rmsnorm_sample_fused")
    return out_ids


def gather_rows(table, ids, out=None, stream=None):
    """out[b] = table[ids[b]] on the device (float32 table [R, D], int32 ids [B])."""
    import torch
    _require_cuda(table, ids, out)
    R, D = table.shape
    B = ids.numel()
    if out is None:
        out = torch.empty(B, D, dtype=torch.float32, device=table.device)
    _check(lib().sampler_gather_rows(_ptr(table), R, D, _ptr(ids), B, _ptr(out), _stream_ptr(stream)),
           "sampler_gather_rows")
    return out


def sample_batched_host(logits_np, temperature, topp, states_np, topp_rows_np=None, probs_in=False):
    """Host-buffer entry point: numpy float32 [B, V] in, int32 ids out; the
    uint64 states array is advanced in place."""
    import numpy as np
    B, V = logits_np.shape
    assert logits_np.dtype == np.float32 and logits_np.flags.c_contiguous
    ids = np.empty(B, dtype=np.int32)
    cfg = SamplerBatchConfig(V, float(temperature), float(topp), SAMPLER_FLAG_PROBS_IN if probs_in else 0)
    tp = None if topp_rows_np is None else topp_rows_np.ctypes.data_as(ctypes.c_void_p)
    st = None if states_np is None else states_np.ctypes.data_as(ctypes.c_void_p)
    rc = lib().sampler_batched_host(ctypes.byref(cfg), logits_np.ctypes.data_as(ctypes.c_void_p), B, V, tp, st,
                                    ids.ctypes.data_as(ctypes.c_void_p))
    _check(rc, "sampler_batched_host")
    return ids


def last_launch_count():
    return lib().sampler_last_launch_count()


# ---- llama2.c surface, for tests that read like the reference's call sites ----
def build_sampler(vocab_size, temperature, topp, rng_seed):
    s = Sampler()
    lib().build_sampler(ctypes.byref(s), vocab_size, temperature, topp, ctypes.c_ulonglong(rng_seed))
    return s


def free_sampler(s):
    lib().free_sampler(ctypes.byref(s))


def sample(s, logits_np, entry="sample"):
    """llama2.c sample(): logits_np (float32, writable) is overwritten with the
    probabilities when temperature != 0.  entry="sample_debug" / "do_sample"
    calls the variants of the reference's CUDA translation units instead."""
    fp = logits_np.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    r = getattr(lib(), entry)(ctypes.byref(s), fp)
    if r < 0:
        raise SamplerError(f"{entry} failed: " + lib().sampler_last_error().decode())
    return r
