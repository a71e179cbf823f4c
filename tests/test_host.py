"""CPU tests of libvkb.so without a GPU: the library loads, exports every entry point its headers declare, rejects
bad arguments before touching CUDA, and its host-side quantiser / packers / generators agree with the oracle."""
import ctypes
import os
import re

import numpy as np
import pytest

import vkb
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for h in ("vkb.h", "vkb_host.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names.update(re.findall(r"\b(vkb_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    L = vkb.lib()
    declared = _declared_symbols()
    assert "vkb_gemv_q4" in declared and "vkb_moe_q4" in declared
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing


def test_c_abi_is_exactly_the_headers():
    """Every unmangled function libvkb.so exports is declared in include/ (no undocumented entry points)."""
    import shutil
    import subprocess
    if shutil.which("nm") is None:
        pytest.skip("nm not available")
    out = subprocess.run(["nm", "-D", "--defined-only", vkb.LIB_PATH], capture_output=True, text=True, check=True)
    exported = {f[2] for f in (ln.split() for ln in out.stdout.splitlines())
                if len(f) == 3 and f[1] == "T" and not f[2].startswith("_")}
    assert exported == set(_declared_symbols()), exported ^ set(_declared_symbols())


def test_every_declared_symbol_has_a_binding():
    """vkb.lib() sets argument and result types for every entry point the headers declare (a ctypes call without them
    would pass 64-bit pointers as C ints)."""
    L = vkb.lib()
    unbound = [n for n in _declared_symbols() if getattr(L, n).argtypes is None]
    assert not unbound, unbound


def test_missing_library_fails_loudly(monkeypatch):
    """No fallback: without libvkb.so every entry point of the Python binding raises instead of computing elsewhere."""
    monkeypatch.setattr(vkb, "_lib", None)
    monkeypatch.setattr(vkb, "LIB_PATH", os.path.join(ROOT, "no-such-dir", "libvkb.so"))
    with pytest.raises(ImportError, match="missing"):
        vkb.lib()
    import torch
    q = torch.zeros(64 * 256 // 2, dtype=torch.uint8)
    s = torch.zeros((64, 256 // 32), dtype=torch.float16)
    x = torch.zeros((1, 256), dtype=torch.float16)
    with pytest.raises(ImportError):
        vkb.gemv(O.FMT_Q4, q, s, x)


def test_strerror_and_version():
    assert vkb.lib().vkb_version() >= 100
    assert "unsupported" in vkb.strerror(vkb.EUNSUPPORTED)
    assert "invalid" in vkb.strerror(vkb.EINVAL)


def test_bad_arguments_rejected_before_any_cuda_call():
    L = vkb.lib()
    nul = ctypes.c_void_p(0)
    one = ctypes.c_void_p(16)
    # null pointers, bad sizes, K not a multiple of 32, too many tokens: nothing launched, no CUDA needed
    assert L.vkb_gemv_q4(nul, one, one, one, 64, 256, 1, nul) == vkb.EINVAL
    assert L.vkb_gemv_q4(one, one, one, one, 0, 256, 1, nul) == vkb.EINVAL
    assert L.vkb_gemv_q4(one, one, one, one, 64, 250, 1, nul) == vkb.EUNSUPPORTED
    assert L.vkb_gemv_q4(one, one, one, one, 64, 256, 9, nul) == vkb.EUNSUPPORTED
    assert L.vkb_gemv_q4(one, one, one, one, 64, 256, 0, nul) == vkb.EINVAL
    assert L.vkb_gemv(7, one, one, one, one, 0, 64, 256, 1, nul) == vkb.EUNSUPPORTED
    assert L.vkb_moe_q4(one, one, nul, 1, 8, one, one, 8, 0, 64, 256, nul) == vkb.EINVAL
    # multi-GPU entry points without a communicator: refused before anything else
    assert L.vkb_gemm_q4_tc_rowsplit_noalloc(nul, one, one, one, one, 1024, 2048, 64, nul) == vkb.ENOCOMM
    assert L.vkb_gemm_q4_tc_rowsplit(nul, one, one, one, one, one, 1024, 2048, 64, nul) == vkb.ENOCOMM
    assert L.vkb_gemm_q4_tc_rowsplit_p2p(nul, one, one, one, one, 1024, 2048, 64, nul) == vkb.ENOCOMM


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2])
def test_pack_matches_oracle(fmt):
    rng = np.random.default_rng(fmt)
    lo, hi = {O.FMT_Q4: (-8, 7), O.FMT_Q8: (-127, 127), O.FMT_Q2: (-2, 1)}[fmt]
    codes = rng.integers(lo, hi + 1, size=(37, 256)).astype(np.int8)
    for sab in (False, True):
        mine = vkb.pack(fmt, codes, sabotage=sab)
        assert np.array_equal(mine.view(np.uint8), O.pack(fmt, codes, sabotage=sab).view(np.uint8)), (fmt, sab)


def test_pack_matches_reference_golden(golden):
    assert np.array_equal(vkb.pack(O.FMT_Q4, golden["a_q4_codes"]), golden["a_q4_packed"])
    assert np.array_equal(vkb.pack(O.FMT_Q4, golden["a_q4_codes"], True), golden["a_q4_packed_sab"])
    assert np.array_equal(vkb.pack(O.FMT_Q2, golden["odd_q2_codes"]), golden["odd_q2_packed"])


@pytest.mark.parametrize("fmt", [O.FMT_Q4, O.FMT_Q8, O.FMT_Q2])
def test_quantize_matches_oracle(fmt):
    w = vkb.synth_normal(0, (64, 512), 0.02)
    w[3, :32] = 0.0                              # an all-zero block
    w[5, 7] = 0.5                                # an outlier
    c1, s1 = vkb.quantize(fmt, w)
    c2, s2 = O.quantize(fmt, w)
    assert np.array_equal(s1, s2)
    assert np.array_equal(c1, c2)


def test_synth_normal_is_deterministic_and_normal():
    a = vkb.synth_normal(0, (1 << 16,), 0.02)
    b = vkb.synth_normal(0, (1 << 16,), 0.02)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 5e-4 and abs(a.std() - 0.02) < 5e-4
    assert not np.array_equal(a, vkb.synth_normal(1, (1 << 16,), 0.02))


def test_synth_topk_distinct():
    idx = vkb.synth_topk(0, 64, 128, 8)
    assert idx.shape == (64, 8) and idx.min() >= 0 and idx.max() < 128
    assert all(len(set(r)) == 8 for r in idx)
    assert np.array_equal(idx, vkb.synth_topk(0, 64, 128, 8))
