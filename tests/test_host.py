"""Host-side logic that needs no GPU: the C ABI library loads and exports what
the header declares, argument validation at the boundary, the quartz drop-in
patching, and the synthetic workload recipes."""

import ctypes
import re
import subprocess
import types
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "quartz_b200.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^int\s+(qz_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from quartz_b200 import _lib
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} not exported"
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (qz_\w+)$", out, flags=re.M))
    assert set(declared) <= exported


def test_ctypes_signatures_match_the_header_prototypes():
    """Every declared prototype and its ctypes binding agree argument by
    argument: pointers with pointers, and each scalar with its C type."""
    from quartz_b200 import _lib
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = re.findall(r"^int\s+(qz_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M | re.S)
    assert len(protos) == len(_declared())
    scalar = {"int64_t": ctypes.c_int64, "int": ctypes.c_int, "size_t": ctypes.c_size_t,
              "float": ctypes.c_float, "uint32_t": ctypes.c_uint32}

    def kind(t):
        if t in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(t, ctypes._Pointer):
            return "ptr"
        return t

    for name, params in protos:
        want = []
        for prm in (x.strip() for x in params.split(",")):
            if not prm or prm == "void":
                continue
            if "*" in prm:
                want.append("ptr")
            else:
                ctype = prm.rsplit(None, 1)[0].replace("const", "").strip()
                assert ctype in scalar, f"{name}: unexpected parameter type {ctype!r}"
                want.append(scalar[ctype])
        got = [kind(t) for t in _lib.SIGNATURES[name][0]]
        assert got == want, f"{name}: ctypes {got} vs header {want}"
        assert _lib.SIGNATURES[name][1] is ctypes.c_int, f"{name}: status return"


def test_version_and_error_buffer():
    from quartz_b200 import _lib
    lib = _lib.load()
    assert lib.qz_version() >= (0 << 16) | (1 << 8)
    assert lib.qz_mlp_workspace_bytes() >= 8


@pytest.mark.parametrize("args,msg", [
    ((1, 1, 3, 1, 1, 4, 64, None, None), "do not tile"),      # K % ng
    ((1, 1, 0, 1, 1, 4, 64, None, None), "ng must be"),       # ng < 1
    ((1, 1, 1, 1, 1, -1, 64, None, None), "negative"),        # N < 0
    ((None, 1, 1, 1, 1, 4, 64, None, None), "null weight"),   # q null
])
def test_gemv_argument_checks_without_gpu(args, msg):
    """Invalid arguments are refused before any CUDA call (no GPU needed)."""
    from quartz_b200 import _lib
    lib = _lib.load()
    rc = lib.qz_gemv_w8(*args)
    assert rc == _lib.QZ_ERR_INVALID
    assert msg in _lib.last_error()
    with pytest.raises(ValueError, match=msg):
        _lib.check(rc)


def test_gemm_and_mlp_argument_checks_without_gpu():
    from quartz_b200 import _lib
    lib = _lib.load()
    assert lib.qz_gemm_w8(1, 1, 1, 1, 1, -2, 4, 64, None, None) == _lib.QZ_ERR_INVALID
    assert "negative M" in _lib.last_error()
    # empty problems are no-ops that touch nothing
    assert lib.qz_gemm_w8(1, 1, 1, 1, 1, 0, 4, 64, None, None) == _lib.QZ_OK
    assert lib.qz_gemv_w8(1, 1, 1, 1, 1, 0, 64, None, None) == _lib.QZ_OK
    rc = lib.qz_fused_mlp_decode(1, 1, 3, 1, 1, 1, 1, 1, 1, None, 64, 128, None, None)
    assert rc == _lib.QZ_ERR_INVALID and "do not tile" in _lib.last_error()


def _fake_quartz():
    mods = {}
    for name in ("quartz.kernels.int8", "quartz.kernels.fused", "quartz.kernels",
                 "quartz.quantize"):
        m = types.ModuleType(name)
        mods[name] = m
    for n in ("w8a32_gemv", "w8a32_gemv_serial", "w8a32_gemm", "matmul_int8", "warmup"):
        setattr(mods["quartz.kernels.int8"], n, f"orig.{n}")
    for n in ("fused_mlp_decode", "warmup_fused"):
        setattr(mods["quartz.kernels.fused"], n, f"orig.{n}")
    for n in ("w8a32_gemv", "w8a32_gemm", "matmul_int8", "warmup"):
        setattr(mods["quartz.kernels"], n, f"orig.{n}")
    for n in ("matmul_int8", "warmup", "fused_mlp_decode", "warmup_fused"):
        setattr(mods["quartz.quantize"], n, f"orig.{n}")
    return mods


def test_install_patches_every_binding_and_uninstalls():
    import quartz_b200
    from quartz_b200 import kernels
    mods = _fake_quartz()
    inst = quartz_b200.install(mods)
    assert mods["quartz.quantize"].matmul_int8 is kernels.matmul_int8      # quantize.py:20
    assert mods["quartz.quantize"].fused_mlp_decode is kernels.fused_mlp_decode  # :21
    assert mods["quartz.kernels.int8"].w8a32_gemv_serial is kernels.w8a32_gemv_serial
    assert mods["quartz.kernels"].matmul_int8 is kernels.matmul_int8
    inst.uninstall()
    assert mods["quartz.quantize"].matmul_int8 == "orig.matmul_int8"
    assert mods["quartz.kernels.fused"].warmup_fused == "orig.warmup_fused"


def test_install_strict_missing_attribute_rolls_back():
    import quartz_b200
    mods = _fake_quartz()
    del mods["quartz.quantize"].warmup_fused
    with pytest.raises(AttributeError):
        quartz_b200.install(mods)
    assert mods["quartz.kernels.int8"].w8a32_gemv == "orig.w8a32_gemv"


def test_workload_recipes_and_byte_model():
    from quartz_b200.workloads import (gemv_algorithmic_bytes, gemv_case, mlp_algorithmic_bytes,
                                       mlp_case)
    assert gemv_algorithmic_bytes(151936, 1024) == 156_802_048
    assert mlp_algorithmic_bytes(1024, 3072) == 9_474_048
    c = gemv_case(64, 32, seed=3)
    assert c.q.dtype == np.int8 and c.scale.shape == (64, 1) and c.x.shape == (1, 32)
    m = mlp_case(32, 64, M=2, seed=4, group_size=32)
    assert m.gu_q.shape == (128, 32) and m.gu_s.shape == (128, 1)
    assert m.down_q.shape == (32, 64) and m.down_s.shape == (32, 2) and m.x.shape == (2, 32)
    # same seed, same bytes
    assert np.array_equal(gemv_case(64, 32, seed=3).q, c.q)


def test_numpy_api_validates_before_touching_the_gpu():
    from quartz_b200 import kernels
    with pytest.raises(ValueError, match="do not tile"):
        kernels.matmul_int8(np.zeros((4, 64), np.int8), np.ones((4, 3), np.float32),
                            np.zeros((1, 64), np.float32))
    with pytest.raises(TypeError):
        kernels.w8a32_gemv(np.zeros((4, 64), np.float32), np.ones((4, 1), np.float32),
                           np.zeros(64, np.float32), np.zeros(4, np.float32))


def test_kernel_resources():
    """ptxas figures of the built library: no register spills, and at most 256
    bytes of static shared memory per kernel (the launch code reserves 256
    bytes below the opt-in maximum for it)."""
    from quartz_b200 import build
    if not build.RESOURCES.exists():
        pytest.skip("library built without resource figures")
    rows = build.RESOURCES.read_text().split("\n")
    bad = [r for r in rows if r and (int(r.split("smem=")[1].split()[0]) > 256
                                     or int(r.split("spill=")[1]) > 0)]
    assert not bad, bad


def test_bench_reference_arm_prints_the_same_config():
    """`bench.py --impl reference` (the CPU port on the host cores) prints one
    JSON line whose config is the dict the repo's own arm prints."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    r = subprocess.run([sys.executable, str(repo / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=repo)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    sys.path.insert(0, str(repo))
    import bench
    assert d["impl"] == "reference"
    assert d["config"] == bench.bench_config(1, 3)
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
