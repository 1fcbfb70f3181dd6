"""The C ABI from a plain C program (tests/c_abi/spark_layer.c): the header and the shared
library are all a C host needs, besides the CUDA runtime.  The CPU test compiles and links
it; the GPU test runs one Spark layer through it and checks the route bit for bit and the
output within the bf16 tolerance against the oracle, and bit for bit against the Python
path over the same library."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
SOURCE = ROOT / "tests" / "c_abi" / "spark_layer.c"
LIBDIR = ROOT / "spark-h3_b200" / "spark_h3_b200" / "_lib"


def _cuda_home() -> Path:
    from torch.utils.cpp_extension import CUDA_HOME

    if CUDA_HOME is None:
        pytest.skip("no CUDA toolkit to build the C program against")
    return Path(CUDA_HOME)


def build_program(out_dir: Path) -> Path:
    if shutil.which("gcc") is None:
        pytest.skip("gcc is not installed")
    if not (LIBDIR / "libsparkh3b200.so").exists():
        pytest.fail("libsparkh3b200.so is not built (python __graft_entry__.py)")
    cuda = _cuda_home()
    exe = out_dir / "spark_layer"
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
           f"-I{cuda / 'include'}", str(SOURCE), f"-L{LIBDIR}", "-lsparkh3b200", f"-L{cuda / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{LIBDIR}:{cuda / 'lib64'}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_program_builds_against_the_header(tmp_path):
    exe = build_program(tmp_path)
    usage = subprocess.run([str(exe)], capture_output=True, text=True)
    assert usage.returncode == 1 and "usage:" in usage.stderr


@pytest.mark.gpu
def test_c_program_runs_a_layer_that_matches_the_oracle(cuda_device, tmp_path):
    from oracle import oracle
    from spark_h3_b200 import ops
    from spark_h3_b200.synthetic import make_qkv

    block, heads = 128, 2
    q, k, v = make_qkv((4, 16, 33), heads, 128, seed=61, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    T = q.shape[1]  # 2112: 16 complete 128-token blocks and a 64-row dense suffix
    topk = ops.target_topk(0.1, T // block)
    for name, t in zip("qkv", (q, k, v)):
        t.contiguous().view(torch.int16).numpy().tofile(tmp_path / f"{name}.bin")
    exe = build_program(tmp_path)
    run = subprocess.run([str(exe), str(T), str(heads), "128", str(block), str(topk), ops.scale_log2(128).hex(),
                          *(str(tmp_path / f"{n}.bin") for n in "qkv"), str(tmp_path)],
                         capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr
    qb, nb = T // block, -(-T // block)
    packed = np.fromfile(tmp_path / "packed.bin", dtype=np.int32).reshape(1, qb, heads, -(-nb // 32))
    indices = np.fromfile(tmp_path / "indices.bin", dtype=np.int32).reshape(1, qb, heads, topk)
    out = torch.from_numpy(np.fromfile(tmp_path / "out.bin", dtype=np.int16).reshape(1, T, heads, 128))
    out = out.view(torch.bfloat16)

    def to_oracle(t):
        return oracle.Tensor(t.contiguous().view(torch.int16).numpy().view(np.uint16), "bfloat16")

    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1)
    np.testing.assert_array_equal(packed, ref["packed"])
    np.testing.assert_array_equal(indices, ref["indices"])
    got = out.float().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref["out"]).max() <= 2e-2  # bf16 attention tolerance
    a, b = got.astype(np.float64).ravel(), ref["out"].astype(np.float64).ravel()
    assert a @ b / (np.linalg.norm(a) * np.linalg.norm(b)) >= 0.9995
    py = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block, topk_ratio=0.1)
    assert torch.equal(py.cpu(), out)
