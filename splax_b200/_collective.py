"""Gradient exchange of a camera-sharded step: the sum over ranks of the fp32 gaussian
gradients, through NVLink SHARP (NVLS) on the NVSwitch fabric.

The reference has no multi-device path; a data-parallel training step over a camera mesh would
psum these gradients (an NCCL all-reduce). Here each rank renders its cameras, copies its
gradients into one symmetric buffer (a copy per rank, one multicast address over all copies,
set up through torch.distributed's symmetric memory), and ``splax_nvls_allreduce_f32`` sums
the buffer in place: each rank reduces its shard with multimem.ld_reduce and multicasts the sums
with multimem.st, between two cross-rank barriers. Every rank ends with identical sums.

One process per GPU; the group's ranks must share an NVSwitch fabric with multicast support.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib

_ALIGN = 64  # floats: the flag array starts 256-byte aligned


class GradAllReduce:
    """Sum all-reduce of a fixed list of fp32 arrays (shapes given once) over a process group.

    ``reduce(tensors)`` copies the tensors into the symmetric buffer, runs the NVLS reduction
    and returns views of the summed buffer with the tensors' shapes; the views stay valid until
    the next call. Raises RuntimeError at construction when the fabric has no multicast.
    """

    def __init__(self, shapes: Sequence[torch.Size | tuple], device: torch.device, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 1 <= self.world <= 8:
            raise RuntimeError("NVLS all-reduce supports 1 to 8 ranks")
        self.shapes = [torch.Size(s) for s in shapes]
        self.sizes = [s.numel() for s in self.shapes]
        self.n = sum(self.sizes)
        n_pad = -(-self.n // _ALIGN) * _ALIGN
        # floats: payload | u64 flags[world] | u32 error word
        total = n_pad + 2 * self.world + _ALIGN
        self.buf = symm_mem.empty(total, dtype=torch.float32, device=device)
        self.buf[n_pad:].zero_()
        torch.cuda.synchronize(device)
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        self.hdl = symm_mem.rendezvous(self.buf, name)
        if not self.hdl.multicast_ptr:
            raise RuntimeError("NVLS all-reduce: this fabric offers no multicast address")
        base = self.hdl.buffer_ptrs[self.rank]
        off = self.buf.data_ptr() - base
        if off < 0 or off + 4 * total > self.hdl.buffer_size:
            raise RuntimeError("NVLS all-reduce: buffer outside its symmetric allocation")
        self.mc = self.hdl.multicast_ptr + off
        flag_off = off + 4 * n_pad
        self.flag_ptrs = (ctypes.c_void_p * self.world)(
            *[self.hdl.buffer_ptrs[q] + flag_off for q in range(self.world)])
        self.err = self.buf[n_pad + 2 * self.world:n_pad + 2 * self.world + 1]
        self.payload = self.buf[:self.n]
        self.views = []
        o = 0
        for s, k in zip(self.shapes, self.sizes):
            self.views.append(self.payload[o:o + k].view(s))
            o += k
        self.epoch = 1
        dist.barrier(group)

    def reduce(self, tensors: Sequence[torch.Tensor]) -> list[torch.Tensor]:
        if len(tensors) != len(self.shapes):
            raise ValueError("reduce: tensor count differs from the shapes given at construction")
        for t, s in zip(tensors, self.shapes):
            if t.shape != s or t.dtype != torch.float32:
                raise ValueError("reduce: tensors must match the construction shapes, fp32")
        torch.cat([t.reshape(-1) for t in tensors], out=self.payload)
        stream = torch.cuda.current_stream(self.buf.device).cuda_stream
        _lib.check(_lib.load().splax_nvls_allreduce_f32(
            ctypes.c_void_p(self.mc), self.flag_ptrs, self.rank, self.world, self.n,
            ctypes.c_uint64(self.epoch), ctypes.c_void_p(self.err.data_ptr()),
            ctypes.c_void_p(stream)))
        self.epoch += 2
        return self.views

    def check(self) -> None:
        """Raise if a barrier of an earlier call gave up waiting (synchronises the stream)."""
        e = int(self.err.view(torch.int32).item())
        if e:
            raise _lib.SplaxDeviceError(f"NVLS all-reduce: a cross-rank barrier timed out (0x{e:x})")

    def close(self) -> None:
        """Wait for every rank before the symmetric buffer can be released."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.buf.device)
        dist.barrier(self.group)
