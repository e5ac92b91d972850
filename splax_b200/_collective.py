"""Gradient exchange of a camera-sharded step: the sum over ranks of the fp32 gaussian
gradients, through NVLink SHARP (NVLS) on the NVSwitch fabric.

The reference has no multi-device path; a data-parallel training step over a camera mesh would
psum these gradients (an NCCL all-reduce). Here each rank renders its cameras, copies its
gradients into one symmetric buffer (a copy per rank, one multicast address over all copies,
set up through torch.distributed's symmetric memory), and ``splax_nvls_allreduce_f32`` sums
the buffer in place: each rank reduces its shard with multimem.ld_reduce and multicasts the sums
with multimem.st, between two cross-rank barriers. Every rank ends with identical sums.

``NvlsAdam`` fuses that exchange with the training step's Adam update
(``splax_nvls_adam_step``): each rank sums its shard of the gradients through the switch,
updates that shard of the parameters with its shard of the moments and multicasts the new
parameters into every rank's copy.

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


class NvlsAdam:
    """Adam for camera-sharded training with the gradient exchange fused into the update.

    The parameters live in a symmetric buffer (``self.params`` are new leaf tensors viewing it:
    train with those). ``step(grads)`` copies the gradients into a second symmetric buffer and
    runs ``splax_nvls_adam_step``: each rank sums its 1/G shard of the gradients through the
    switch, updates that shard with its 1/G of the moments (optax.adam's update, as ``Adam``),
    and multicasts the new parameters into every rank's copy. The optimiser state is sharded over
    the ranks; every rank ends the step with identical parameters.
    """

    def __init__(self, params: Sequence[torch.Tensor], lrs: Sequence[float] | float,
                 device: torch.device, group=None, b1: float = 0.9, b2: float = 0.999,
                 eps: float = 1e-8):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        params = list(params)
        if isinstance(lrs, (int, float)):
            lrs = [float(lrs)] * len(params)
        if not 1 <= len(params) <= 8 or len(lrs) != len(params):
            raise ValueError("1 to 8 parameter tensors, one learning rate each")
        self.grads = GradAllReduce([p.shape for p in params], device, group)
        self.rank, self.world, self.group = self.grads.rank, self.grads.world, group
        n = self.grads.n
        self.n = n
        self.pbuf = symm_mem.empty(-(-n // _ALIGN) * _ALIGN, dtype=torch.float32, device=device)
        with torch.no_grad():
            torch.cat([p.detach().reshape(-1).to(torch.float32) for p in params],
                      out=self.pbuf[:n])
        torch.cuda.synchronize(device)
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        self.phdl = symm_mem.rendezvous(self.pbuf, name)
        if not self.phdl.multicast_ptr:
            raise RuntimeError("NVLS Adam: this fabric offers no multicast address")
        off = self.pbuf.data_ptr() - self.phdl.buffer_ptrs[self.rank]
        if off < 0 or off + 4 * self.pbuf.numel() > self.phdl.buffer_size:
            raise RuntimeError("NVLS Adam: buffer outside its symmetric allocation")
        self.pmc = self.phdl.multicast_ptr + off
        self.params = []
        o = 0
        for p in params:
            k = p.numel()
            self.params.append(self.pbuf[o:o + k].view(p.shape).requires_grad_())
            o += k
        lib = _lib.load()
        ln = ctypes.c_int64(0)
        _lib.check(lib.splax_nvls_adam_shard_len(n, self.rank, self.world, ctypes.byref(ln)))
        self.exp_avg = torch.zeros(max(ln.value, 4), dtype=torch.float32, device=device)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        self.sizes = (ctypes.c_int64 * len(params))(*[p.numel() for p in params])
        self.lrs = (ctypes.c_float * len(params))(*[float(x) for x in lrs])
        self.b1, self.b2, self.eps = float(b1), float(b2), float(eps)
        self.count = 0
        dist.barrier(group)

    @torch.no_grad()
    def step(self, grads: Sequence[torch.Tensor] | None = None) -> None:
        if grads is None:
            grads = [p.grad for p in self.params]
        torch.cat([g.reshape(-1) for g in grads], out=self.grads.payload)
        self.count += 1
        g = self.grads
        stream = torch.cuda.current_stream(self.pbuf.device).cuda_stream
        _lib.check(_lib.load().splax_nvls_adam_step(
            ctypes.c_void_p(g.mc), ctypes.c_void_p(self.pmc), ctypes.c_void_p(self.pbuf.data_ptr()),
            ctypes.c_void_p(self.exp_avg.data_ptr()), ctypes.c_void_p(self.exp_avg_sq.data_ptr()),
            self.n, len(self.params), self.sizes, self.lrs, self.count, self.b1, self.b2,
            self.eps, g.flag_ptrs, self.rank, self.world, ctypes.c_uint64(g.epoch),
            ctypes.c_void_p(g.err.data_ptr()), ctypes.c_void_p(stream)))
        g.epoch += 2

    def check(self) -> None:
        self.grads.check()

    def close(self) -> None:
        self.grads.close()
