"""The reference's host ABI (include/session.h, buffer.h, dispatch.h) seen
from Python through ctypes: the same structs, the same entry points, the same
call sequence as src/compute.c:51-210 (createSession, createBuffer,
createTransferAndCopy, execute, getExecutionTime, readBuffer, destroyBuffer).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import lib

MEMORY_RAM = 0
MEMORY_VRAM = 1
MAX_OP_BUFFERS = 16
MAX_PUSH_CONSTANTS = 8


class VkMemoryRequirements(C.Structure):
    _fields_ = [("size", C.c_uint64), ("alignment", C.c_uint64), ("memoryTypeBits", C.c_uint32)]


class Device(C.Structure):  # include/device.h
    _fields_ = [("instance", C.c_void_p), ("device", C.c_void_p), ("queue", C.c_void_p),
                ("physicalDevice", C.c_void_p)]


class Buffer(C.Structure):  # include/buffer.h
    _fields_ = [("buffer", C.c_void_p), ("memReqs", VkMemoryRequirements), ("memory", C.c_void_p),
                ("stagingBuffer", C.c_void_p), ("stagingMemory", C.c_void_p),
                ("mappedMemory", C.c_void_p), ("size", C.c_int64), ("memoryType", C.c_int)]


class Session(C.Structure):  # include/session.h
    _fields_ = [("dev", Device), ("pool", C.c_void_p), ("buffer", C.c_void_p), ("fence", C.c_void_p),
                ("qpool", C.c_void_p)]


class Operation(C.Structure):  # include/dispatch.h
    _fields_ = [("shader", C.c_char * 128), ("buffers", Buffer * MAX_OP_BUFFERS), ("bufferCount", C.c_int),
                ("pushConstants", C.c_int * MAX_PUSH_CONSTANTS), ("pushConstantCount", C.c_int),
                ("dispatchX", C.c_int), ("dispatchY", C.c_int), ("dispatchZ", C.c_int)]


_declared = False


def abi() -> C.CDLL:
    """libvkcompute with the reference-ABI entry points declared."""
    global _declared
    L = lib()
    if not _declared:
        P = C.c_void_p
        L.createSession.restype, L.createSession.argtypes = Session, []
        L.destroySession.restype, L.destroySession.argtypes = None, [Session]
        L.createBuffer.restype, L.createBuffer.argtypes = Buffer, [P, P, P, C.c_int64, C.c_int]
        L.createTransferAndCopy.restype = None
        L.createTransferAndCopy.argtypes = [P, P, C.POINTER(Buffer), C.c_int]
        L.readBuffer.restype, L.readBuffer.argtypes = None, [P, P, P, Buffer, P]
        L.writeBuffer.restype, L.writeBuffer.argtypes = None, [P, P, Buffer, P]
        L.destroyBuffer.restype, L.destroyBuffer.argtypes = None, [P, Buffer]
        L.execute.restype, L.execute.argtypes = None, [Session, C.POINTER(Operation), C.c_int]
        L.getExecutionTime.restype, L.getExecutionTime.argtypes = C.c_double, [Session]
        _declared = True
    return L


def create_session() -> Session:
    return abi().createSession()


def create_buffer(s: Session, data: np.ndarray | None, size: int | None = None,
                  memory_type: int = MEMORY_RAM) -> Buffer:
    if data is not None:
        data = np.ascontiguousarray(data)
        size = data.nbytes if size is None else size
        ptr = data.ctypes.data_as(C.c_void_p)
    else:
        ptr = None
    return abi().createBuffer(s.dev.device, s.dev.physicalDevice, ptr, int(size), memory_type)


def read_buffer(s: Session, b: Buffer, dtype=np.float32) -> np.ndarray:
    out = np.empty(b.size // np.dtype(dtype).itemsize, dtype=dtype)
    abi().readBuffer(s.dev.device, s.dev.physicalDevice, s.dev.queue, b, out.ctypes.data_as(C.c_void_p))
    return out


def write_buffer(s: Session, b: Buffer, data: np.ndarray) -> None:
    data = np.ascontiguousarray(data)
    assert data.nbytes >= b.size
    abi().writeBuffer(s.dev.device, s.dev.queue, b, data.ctypes.data_as(C.c_void_p))


def destroy_buffer(s: Session, b: Buffer) -> None:
    abi().destroyBuffer(s.dev.device, b)


def operation(shader: str, buffers: list[Buffer], push: list[int], dispatch=(1, 1, 1)) -> Operation:
    op = Operation()
    op.shader = shader.encode()
    for i, b in enumerate(buffers):
        op.buffers[i] = b
    op.bufferCount = len(buffers)
    for i, v in enumerate(push):
        op.pushConstants[i] = int(v)
    op.pushConstantCount = len(push)
    op.dispatchX, op.dispatchY, op.dispatchZ = dispatch
    return op


def execute(s: Session, ops: list[Operation]) -> float:
    """Runs the operations in order and returns getExecutionTime (ms)."""
    arr = (Operation * len(ops))(*ops)
    abi().execute(s, arr, len(ops))
    return abi().getExecutionTime(s)


def destroy_session(s: Session) -> None:
    abi().destroySession(s)
