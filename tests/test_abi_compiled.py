"""The boundary compiled, not just bound through ctypes.

1. A plain C program (tests/abi_c_check.c) calls the C ABI of include/crosslane_b200.h
   directly: host-only entry points, error codes and messages, null handles; on a GPU box
   (`-m gpu` variant) it also creates and queries a bank.
2. The C++ adapter include/crosslane_b200_warm.hpp (the CUDA lane as crosslane's
   WarmRedirect) is compiled against crosslane's own engine/strata/warm/runtime.hpp with
   STRATA_FORK_WARM, as the engine builds it, including a translation unit that registers
   it with warm_register: every override must match the reference's virtual signatures.
   The checkout is taken from the --crosslane-ref pytest option, CROSSLANE_REF, or the
   checkout oracle/_ref was built from (oracle/_ref/checkout); the test is skipped where no
   checkout exists (the GPU boxes).
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
LIB_DIR = os.path.join(ROOT, "crosslane_b200")


def _build_c_check(tmp_path):
    exe = str(tmp_path / "abi_c_check")
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", INCLUDE, os.path.join(ROOT, "tests", "abi_c_check.c"),
           "-L", LIB_DIR, "-lcrosslane_b200", f"-Wl,-rpath,{LIB_DIR}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_caller_without_gpu(tmp_path):
    exe = _build_c_check(tmp_path)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")  # no device: bank creation must fail cleanly
    r = subprocess.run([exe], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0 and "abi ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_c_caller_with_gpu(tmp_path, cuda):
    exe = _build_c_check(tmp_path)
    r = subprocess.run([exe, "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "abi ok" in r.stdout, r.stdout + r.stderr


def _crosslane_ref(request):
    ref = request.config.getoption("--crosslane-ref") or os.environ.get("CROSSLANE_REF")
    recorded = os.path.join(ROOT, "oracle", "_ref", "checkout")
    if not ref and os.path.isfile(recorded):
        with open(recorded) as f:
            ref = f.read().strip()
    if not ref or not os.path.isfile(os.path.join(ref, "engine", "strata", "warm", "runtime.hpp")):
        pytest.skip("no crosslane checkout (set CROSSLANE_REF or --crosslane-ref)")
    return ref


def test_warm_adapter_compiles_against_crosslane(request, tmp_path):
    ref = _crosslane_ref(request)
    if shutil.which("g++") is None:
        pytest.skip("no C++ compiler")
    tu = tmp_path / "register_cuda_lane.cpp"
    tu.write_text(
        '#include "crosslane_b200_warm.hpp"\n'
        "#include <memory>\n"
        "namespace strata::wiring {\n"
        "void register_cuda_lane(const clb_bank_config_v1& cfg) {\n"
        "    static std::unique_ptr<CudaBank> lane = std::make_unique<CudaBank>(cfg);\n"
        "    WarmRedirect* base = lane.get();\n"
        "    warm_register(base, true);\n"
        "}\n"
        "static_assert(!std::is_abstract_v<CudaBank>, \"every pure virtual of WarmRedirect is implemented\");\n"
        "}\n")
    cmd = ["g++", "-std=c++20", "-fsyntax-only", "-Wall", "-Wextra", "-Werror", "-DSTRATA_FORK_WARM",
           "-isystem", os.path.join(ref, "engine", "strata", "warm"), "-I", INCLUDE, str(tu)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
