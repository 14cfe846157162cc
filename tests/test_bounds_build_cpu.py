"""The bounds-checked build variant (DMAD_BOUNDS_CHECK=1) of the peer-memory kernels still compiles.

The guards record status code 6 and skip the access instead of faulting; release builds compile them
out, so this test keeps the guarded variant from rotting.  Needs only nvcc (no GPU)."""
import os
import shutil
import subprocess
import sysconfig

import pytest

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = shutil.which("nvcc") or ("/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else None)


@pytest.mark.skipif(NVCC is None, reason="nvcc not available")
def test_guarded_kernels_compile(tmp_path):
    from torch.utils.cpp_extension import include_paths

    inc = sum((["-I", p] for p in include_paths(device_type="cuda") + [os.path.join(HERE, "csrc"),
                                                                       sysconfig.get_paths()["include"]]), [])
    procs = {}
    for src in ("cp_a2a.cu", "fsdp.cu"):  # both compiles run at once
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O1", "-DDMAD_BOUNDS_CHECK=1",
               "--expt-relaxed-constexpr", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
               "-DTORCH_EXTENSION_NAME=_C", "-D_GLIBCXX_USE_CXX11_ABI=1", *inc, "-c",
               os.path.join(HERE, "csrc", src), "-o", str(tmp_path / (src + ".o"))]
        procs[src] = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    for src, p in procs.items():
        _, err = p.communicate(timeout=900)
        assert p.returncode == 0, f"{src}: {err[-3000:]}"
