"""Receive buffers and arrival counters for the fused tensor-parallel all-gather.

Every rank allocates one block of exchange memory with the library
(``fqkv_ipc_alloc``: zero-filled, with a CUDA IPC handle), the handles are
swapped with ``torch.distributed.all_gather_object`` and every rank maps the
others' blocks (``fqkv_ipc_open``).  Layout of a block::

    [0, 8*world)          arrival counters, slot r counts outputs received from rank r
    [256, 264)            this rank's wait sequence number
    [512 + l*LB, ...)     layer l receive buffer: [world, B, Hq_local, D] fp16

The decode kernel of layer l stores rank r's [B, Hq_local, D] attention
output into slice r of the layer-l buffer of *every* rank over NVLink and
counts its output units on every rank's slot r; ``wait(l)`` then blocks the
stream until all slots reached this call's count.  One buffer per layer: a
rank can run at most one layer ahead of the slowest rank (each layer waits
for everybody's previous layer), so a layer's buffer is never rewritten while
a peer still reads it.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native, ops

__all__ = ["PeerExchange"]

_ALIGN = 256
_BUF0 = 512


class _DevArray:
    """Minimal ``__cuda_array_interface__`` view of device memory owned elsewhere."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str = "<f2"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


def _check(rc: int, what: str) -> None:
    _native.check(rc, what)


class PeerExchange:
    """This rank's view of every rank's exchange block (see the module docstring)."""

    def __init__(self, group, layers: int, batch: int, heads_local: int, head_dim: int, device: torch.device):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= _native.TP_MAX_RANKS:
            raise ValueError(f"tensor-parallel exchange supports 2..{_native.TP_MAX_RANKS} ranks")
        self.device = device
        self.layers = layers
        self.slice_elems = batch * heads_local * head_dim
        self.shape = (self.world, batch, heads_local, head_dim)
        self.layer_bytes = -(-self.world * self.slice_elems * 2 // _ALIGN) * _ALIGN
        self.nbytes = _BUF0 + layers * self.layer_bytes
        lib = _native.lib()
        with torch.cuda.device(device):
            ptr = ctypes.c_void_p()
            handle = (ctypes.c_ubyte * 64)()
            _check(lib.fqkv_ipc_alloc(self.nbytes, ctypes.byref(ptr), handle), "ipc_alloc")
            self.base = int(ptr.value)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.peers = []
            try:
                for r, h in enumerate(handles):
                    if r == self.rank:
                        self.peers.append(self.base)
                        continue
                    p = ctypes.c_void_p()
                    buf = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                    _check(lib.fqkv_ipc_open(buf, ctypes.byref(p)), f"ipc_open (rank {r})")
                    self.peers.append(int(p.value))
            except Exception:
                # undo this rank's mappings and memory; the other ranks' waits on this rank
                # then end with device status 64 instead of hanging
                for r, p in enumerate(self.peers):
                    if r != self.rank:
                        lib.fqkv_ipc_close(ctypes.c_void_p(p))
                lib.fqkv_ipc_free(ctypes.c_void_p(self.base))
                raise
        self.counters = self.base
        self.sequence = self.base + _ALIGN
        self.tp_out = []
        self.views = []
        for l in range(layers):
            t = _native.TpOut()
            t.world, t.rank, t.dst_offset = self.world, self.rank, self.rank * self.slice_elems
            for p, pb in enumerate(self.peers):
                t.dst[p] = pb + _BUF0 + l * self.layer_bytes
                t.counters[p] = pb
            self.tp_out.append(t)
            self.views.append(torch.as_tensor(_DevArray(self.base + _BUF0 + l * self.layer_bytes, self.shape),
                                              device=device))
        self.per_call = None
        self.closed = False

    def set_plan(self, kv_format: int, B: int, Hq: int, Hkv: int, max_len: int, D: int, workspace_bytes: int):
        """Arrivals one decode call counts per slot (identical on every rank)."""
        n = int(_native.lib().fqkv_tp_arrivals(kv_format, B, Hq, Hkv, max_len, D, workspace_bytes))
        if n <= 0:
            raise RuntimeError(f"tp_arrivals: bad plan ({n})")
        self.per_call = n

    def wait(self) -> None:
        """Block the current stream until every rank's output of the current call has arrived."""
        ops.tp_wait(self.counters, self.world, self.per_call, self.sequence, self.device)

    def gathered(self, layer: int) -> torch.Tensor:
        """[world, B, Hq_local, D] fp16 view of the layer's receive buffer on this rank."""
        return self.views[layer]

    def close(self) -> None:
        """Unmap the peers' blocks and free this rank's block (collective: every rank calls it)."""
        import torch.distributed as dist

        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _native.lib()
        with torch.cuda.device(self.device):
            for r, p in enumerate(self.peers):
                if r != self.rank:
                    _check(lib.fqkv_ipc_close(ctypes.c_void_p(p)), "ipc_close")
            dist.barrier(group=self.group)
            _check(lib.fqkv_ipc_free(ctypes.c_void_p(self.base)), "ipc_free")
        self.views = []
        self.closed = True
