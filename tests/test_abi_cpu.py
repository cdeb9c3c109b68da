"""The C-ABI library loads on a host without a GPU and exports every entry
point that include/morph_b200.h declares (no compute calls here)."""
import ctypes
import os
import re

import pytest

from morph_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(REPO, "include", "morph_b200.h")).read()
    return sorted(set(re.findall(r"MB_API\s+[\w\s\*]+?\b(mb_\w+)\s*\(", text)))


def test_header_declares_the_bound_surface():
    declared = declared_symbols()
    assert declared, "no MB_API declarations found"
    assert set(declared) == set(_lib.SIGNATURES), (set(declared) ^ set(_lib.SIGNATURES))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
        assert ctypes.cast(getattr(L, name), ctypes.c_void_p).value


def test_host_only_entry_points():
    L = _lib.lib()
    assert L.mb_version() >= 1
    assert _lib.status_string(_lib.MB_ERR_NONFINITE).startswith("nonfinite gradient")
    st = _lib.StepState()
    assert L.mb_step_state_init(ctypes.byref(st), 65536.0, 2000) == 0
    assert st.scale == 65536.0 and st.growth_interval == 2000 and st.clip_coef == 1.0
    assert L.mb_step_state_init(ctypes.byref(st), 0.0, 2000) == _lib.MB_ERR_ARG
    segs = (_lib.Segment * 3)()
    for i, n in enumerate((1, 2048, 2049)):
        segs[i].w = segs[i].m = segs[i].v = segs[i].g = 4096
        segs[i].numel = n
    tiles = ctypes.c_int64(0)
    assert L.mb_segments_plan(segs, 3, ctypes.byref(tiles)) == 0
    assert [s.tile_begin for s in segs] == [0, 1, 2] and tiles.value == 4
    assert L.mb_workspace_bytes(10) % 256 == 0


def test_status_codes_map_to_reference_exceptions():
    with pytest.raises(FloatingPointError):
        _lib.check(_lib.MB_ERR_OVERFLOW_MIN_SCALE)
    with pytest.raises(FloatingPointError):
        _lib.check(_lib.MB_ERR_NONFINITE)
    with pytest.raises(ValueError):
        _lib.check(_lib.MB_ERR_ARG)
    with pytest.raises(IndexError):
        _lib.check(_lib.MB_ERR_INDEX)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.MB_ERR_CUDA)


def test_c_caller_links_and_runs(tmp_path):
    """A plain C program including the header and linking the library (no
    Python in the loop) runs the host-only entry points and argument checks."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    libdir = os.path.join(repo, "morph_b200")
    exe = tmp_path / "abi_host"
    cuda_lib = "/usr/local/cuda/lib64"
    cmd = [gcc, "-std=c11", "-Wall", "-Werror", os.path.join(here, "c", "abi_host.c"), "-I", os.path.join(repo, "include"),
           "-L", libdir, "-lmorph_b200", f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{cuda_lib}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "c abi ok" in r.stdout


def test_fault_arming_is_host_only_and_validated():
    """The test-only fault entry arms and disarms on the host without touching
    a device; it refuses unknown kernels, negative units and bounds outside
    1 us .. 2 s, and disarming (kernel 0) always succeeds."""
    L = _lib.lib()
    assert L.mb_debug_arm_fault(3, 0, 5_000_000) == _lib.MB_ERR_ARG
    assert L.mb_debug_arm_fault(_lib.MB_FAULT_APPLY, -1, 5_000_000) == _lib.MB_ERR_ARG
    assert L.mb_debug_arm_fault(_lib.MB_FAULT_STATS, 0, 999) == _lib.MB_ERR_ARG
    assert L.mb_debug_arm_fault(_lib.MB_FAULT_GEMM, 0, 2_000_000_001) == _lib.MB_ERR_ARG
    for kernel in (_lib.MB_FAULT_APPLY, _lib.MB_FAULT_STATS, _lib.MB_FAULT_GEMM):
        assert L.mb_debug_arm_fault(kernel, 7, 5_000_000) == _lib.MB_OK
    assert L.mb_debug_arm_fault(0, -1, 0) == _lib.MB_OK


def test_muon_args_layout_and_sm_cap_validation():
    """mb_muon_args as Python binds it (skip pointer, then the SM cap), and a
    negative max_sms is refused before anything reaches a device (the pointers
    here are never dereferenced)."""
    assert ctypes.sizeof(_lib.MuonArgs) == 56
    assert _lib.MuonArgs.skip.offset == 40 and _lib.MuonArgs.max_sms.offset == 48
    L = _lib.lib()
    rows, cols = 256, 512
    nbytes = L.mb_muon_batch_workspace_bytes(1, rows, cols)
    assert nbytes > 0
    fake = (ctypes.c_void_p * 1)(4096)
    args = _lib.MuonArgs(.05, .95, 3.4445, -4.775, 2.0315, 5, 1.0, 1.0, -1e-3, _lib.MB_BF16, None, -1)
    rc = L.mb_muon_step_batched(fake, fake, fake, _lib.MB_BF16, None, _lib.MB_NONE, 1, rows, cols,
                                ctypes.byref(args), 4096, nbytes, None, None)
    assert rc == _lib.MB_ERR_ARG
