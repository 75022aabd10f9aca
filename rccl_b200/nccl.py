"""NCCL communicators for the C entry points rsort_dist_pairs /
rsort_dist_pairs_rank (ctypes over libnccl.so.2).

The library takes ncclComm_t handles from its caller, exactly as a Rust or C
host would pass them.  This module creates them from Python: one
communicator per device of this process (ncclCommInitAll), or one per rank of
a torch.distributed process group (ncclGetUniqueId on rank 0, broadcast over
the group, ncclCommInitRank on every rank).  Import torch first, so that the
NCCL library torch loaded is the one used here and in librsort_b200.so.
"""
from __future__ import annotations

import ctypes
from typing import List, Sequence

_lib = None
UNIQUE_ID_BYTES = 128


class UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_ubyte * UNIQUE_ID_BYTES)]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        import torch  # noqa: F401  (loads torch's NCCL first)
        h = ctypes.CDLL("libnccl.so.2")
        vp, i = ctypes.c_void_p, ctypes.c_int
        h.ncclGetUniqueId.argtypes = [ctypes.POINTER(UniqueId)]
        h.ncclGetUniqueId.restype = i
        h.ncclCommInitRank.argtypes = [ctypes.POINTER(vp), i, UniqueId, i]
        h.ncclCommInitRank.restype = i
        h.ncclCommInitAll.argtypes = [ctypes.POINTER(vp), i, ctypes.POINTER(i)]
        h.ncclCommInitAll.restype = i
        h.ncclCommDestroy.argtypes = [vp]
        h.ncclCommDestroy.restype = i
        h.ncclGetErrorString.argtypes = [i]
        h.ncclGetErrorString.restype = ctypes.c_char_p
        _lib = h
    return _lib


def _check(r: int, what: str) -> None:
    if r != 0:
        raise RuntimeError(f"{what}: {lib().ncclGetErrorString(r).decode()}")


def comm_init_all(devices: Sequence[int]) -> List[int]:
    """One communicator per listed device, all driven from this thread."""
    n = len(devices)
    comms = (ctypes.c_void_p * n)()
    devs = (ctypes.c_int * n)(*devices)
    _check(lib().ncclCommInitAll(comms, n, devs), "ncclCommInitAll")
    return [c for c in comms]


def comm_init_group(group=None) -> int:
    """This rank's communicator over a torch.distributed process group (the
    current CUDA device must be the rank's device)."""
    import torch
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    uid = UniqueId()
    if rank == 0:
        _check(lib().ncclGetUniqueId(ctypes.byref(uid)), "ncclGetUniqueId")
    buf = torch.tensor(list(uid.internal), dtype=torch.uint8,
                       device=torch.device("cuda", torch.cuda.current_device()))
    dist.broadcast(buf, 0, group=group)
    data = bytes(buf.cpu().tolist())
    ctypes.memmove(ctypes.addressof(uid), data, UNIQUE_ID_BYTES)
    comm = ctypes.c_void_p()
    _check(lib().ncclCommInitRank(ctypes.byref(comm), world, uid, rank), "ncclCommInitRank")
    return comm.value


def comm_destroy(comm: int) -> None:
    if comm:
        _check(lib().ncclCommDestroy(ctypes.c_void_p(comm)), "ncclCommDestroy")
