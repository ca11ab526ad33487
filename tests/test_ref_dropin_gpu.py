"""The reference's own driver -- src/compute.c and src/main.c, unmodified,
compiled by oracle/build_ref.sh against include/ and linked to libvkcompute --
runs on the GPU and prints the reference's output line.  Its GPU value
(RmsNorm-swiglu-ffn-FP16 at index 10, compute.c:171-180) must match the
oracle, and its CPU value (compute.c:221-226, the reference's own CPU code)
pins the oracle's data generation and RmsNorm-GEMV formula."""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import pyoracle as o

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
K, N, IDX = 4096, 12288, 10


def run_binary(name):
    exe = REF_DIR / name
    if not exe.exists():
        pytest.skip(f"{exe} not built (oracle/build_ref.sh needs the vk-compute sources)")
    p = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr
    m = re.search(r"Output from index 10: (\S+) (\S+)", p.stdout)
    t = re.search(r"Shader execution time: (\S+) ms", p.stdout)
    assert m and t, p.stdout
    return float(m.group(1)), float(m.group(2)), float(t.group(1))


@pytest.fixture(scope="module")
def expected():
    x = o.get_data(4321, 1, K).ravel()
    g = o.get_data(58923, 1, K).ravel()
    gate = (o.get_data_fp16(936, K, N), None, None)
    up = (o.get_data_fp16(1348, K, N), None, None)
    o.set_threads(8)
    h = o.qswiglu(x, g, gate, up, 16, K, N, 4096, 1e-5)
    # src/compute.c:221-226: rms = sqrt(sum x^2 / K) + 1e-5 on the fp32 weight
    w = o.get_data(936, K, N)[:, IDX].astype(np.float64)
    rms = np.sqrt(np.sum(x.astype(np.float64) ** 2) / K) + 1e-5
    cpu = float(np.sum(x.astype(np.float64) * g / rms * w))
    return h[IDX], cpu


@pytest.mark.parametrize("name", ["ref_dropin", "ref_dropin_lib"])
def test_reference_driver(name, expected):
    gpu, cpu, ms = run_binary(name)
    h10, cpu_ref = expected
    assert ms > 0.0
    # printed with %f (6 decimals)
    assert abs(gpu - h10) <= 2e-3 * max(abs(h10), 1.0), (gpu, h10)
    assert abs(cpu - cpu_ref) <= 1e-4 * max(abs(cpu_ref), 1.0) + 1e-6, (cpu, cpu_ref)
