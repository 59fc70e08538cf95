"""CPU: the C-ABI library loads, exports every symbol include/*.h declares,
and its host-only pieces (xorshift, sharding, Sampler bookkeeping) behave like
the reference.  No device compute is called here."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def built(pkg):
    if not os.path.exists(pkg.library_path()):
        import __graft_entry__
        __graft_entry__.build()
    return pkg


def header_functions():
    text = open(os.path.join(ROOT, "include", "b200_sampler.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "while", "defined")))


def test_header_lists_match(built):
    assert header_functions() == sorted(built.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(built):
    out = subprocess.run(["nm", "-D", "--defined-only", built.library_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in header_functions() if s not in exported]
    assert not missing, missing
    L = built.lib()
    for s in header_functions():
        assert getattr(L, s) is not None


def test_sampler_struct_layout(built):
    assert ctypes.sizeof(built.Sampler) == 32 and ctypes.sizeof(built.ProbIndex) == 8
    s = built.build_sampler(32000, 0.7, 0.9, 1234)
    assert (s.vocab_size, round(s.temperature, 6), round(s.topp, 6), s.rng_state) == (32000, 0.7, 0.9, 1234)
    assert bool(s.probindex)
    built.free_sampler(s)


def test_xorshift_matches_oracle(built, orc):
    L = built.lib()
    st = ctypes.c_ulonglong(42)
    for _ in range(1000):
        c_ref, _ = orc.coin(st.value)
        assert L.random_f32(ctypes.byref(st)) == c_ref


def test_shard_rows_cover_batch(built):
    for batch in (0, 1, 7, 4096, 4097):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                b, c = built.shard_rows(batch, world, r)
                rows.extend(range(b, b + c))
            assert rows == list(range(batch))


def test_device_calls_fail_loudly_without_gpu(built):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    x = np.zeros(16, dtype=np.float32)
    r = built.lib().sample_argmax(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 16)
    assert r == -1
    assert built.lib().sampler_last_error()
