"""libvkcompute.so loads on a machine without a GPU and exports every
function that include/*.h declares (no compute call is made)."""
import re
from pathlib import Path

import pytest

from vk_compute_b200._lib import lib

INCLUDE = Path(__file__).resolve().parents[1] / "include"
DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\([^;{]*\)\s*;", re.M)


def declared_functions():
    names = set()
    for h in INCLUDE.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//.*", "", text)
        for m in DECL.finditer(text):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_reference_abi():
    names = set(declared_functions())
    for fn in ("createSession", "destroySession", "createBuffer", "createTransferAndCopy", "readBuffer",
               "destroyBuffer", "execute", "getExecutionTime", "createDevice", "destroyDevice",
               "createPipeline", "destroyPipeline", "createDescriptor", "destroyDescriptor",
               "createCommand", "destroyCommand", "createFence", "getData", "getDataFP16", "getDataINT8",
               "getDataINT4", "transpose", "transpose_block16", "free_quantized_data"):
        assert fn in names, fn


@pytest.mark.parametrize("name", declared_functions())
def test_symbol_exported(name):
    assert hasattr(lib(), name), f"libvkcompute.so does not export {name}"


REFERENCE_SHADERS = [
    "GEMV-FP16.spv", "GEMV-INT8.spv", "GEMV-INT4.spv", "GEMV.spv", "RmsNorm-GEMV.spv",
    "RmsNorm-GEMV-FP16.spv", "RmsNorm-GEMV-INT8.spv", "RmsNorm-GEMV-INT4.spv",
    "RmsNorm-GEMV-Rope-FP16.spv", "RmsNorm-GEMV-Rope-INT8.spv", "RmsNorm-GEMV-Rope-INT4.spv",
    "RmsNorm-swiglu-ffn.spv", "RmsNorm-swiglu-ffn-FP16.spv", "RmsNorm-swiglu-ffn-INT8.spv",
    "RmsNorm-swiglu-ffn-INT4.spv", "Att-full-FP16.spv", "gemm.spv", "bin/GEMV-INT4.spv", "RmsNorm.spv",
    "gemv1.spv", "gemv2.spv", "gemv3.spv", "gemv4.spv", "gemv5.spv", "gemv6.spv", "gemv7.spv",
    "shader\\gemm.comp",
]


@pytest.mark.parametrize("shader", REFERENCE_SHADERS)
def test_operator_registered(shader):
    assert lib().vkc_has_operator(shader.encode()) == 1


def test_unknown_operator():
    assert lib().vkc_has_operator(b"RmsNorm-QKV-score-V.spv") == 0


def test_wait_limits_outlast_each_other():
    """The collecting CTA of a split-K cluster waits (on the GPU clock) at
    least ten times as long as any peer wait that can hold a depositing CTA
    back, so it never exits while a deposit into its shared memory is still
    to come; both are finite, so no device wait is unbounded."""
    import ctypes as C

    peer, cluster = C.c_uint64(), C.c_uint64()
    lib().vkc_wait_limits(C.byref(peer), C.byref(cluster))
    assert 0 < peer.value <= 1_000_000_000
    assert cluster.value >= 10 * peer.value
    assert cluster.value <= 10_000_000_000


def test_peer_input_layout_matches_header():
    """ops.PeerInput mirrors vkc_peer_input (two pointers, then rank and world)."""
    import ctypes as C

    from vk_compute_b200.ops import PeerInput

    assert C.sizeof(PeerInput) == 2 * C.sizeof(C.c_void_p) + 2 * C.sizeof(C.c_int)
    assert [f[0] for f in PeerInput._fields_] == ["slots", "save", "rank", "world"]
    assert PeerInput.rank.offset == 2 * C.sizeof(C.c_void_p)
