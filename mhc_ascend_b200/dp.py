"""Data-parallel gradient synchronisation for mHC layers.

The mHC layer is independent per token, so data parallelism shards the token
(batch) dimension across GPUs and needs exactly one exchange per step: a sum
of the parameter gradients (phi_pre/post/res, rmsnorm_weight, alpha x3,
b x3 -- about 1.6 MB at n=4, C=4096).  ``GradBucket`` packs them into one
flat buffer (fp32 for the layer's parameters) in a fixed parameter order and all-reduces it with a single
collective (NCCL over NVLink on GPUs, gloo on CPU), then scatters the result
back.  The reference has no multi-device support (single-NPU library).
"""

from __future__ import annotations

from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


class GradBucket:
    """One flat all-reduce bucket over a fixed list of parameters."""

    def __init__(self, params: Iterable[torch.nn.Parameter], average: bool = True):
        self.params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        self.average = average
        self.numel = sum(p.numel() for p in self.params)
        dtypes = {p.dtype for p in self.params}
        # one dtype for the whole bucket: the parameters' own when uniform
        self.dtype = dtypes.pop() if len(dtypes) == 1 else torch.float32
        self._flat: Optional[torch.Tensor] = None

    def _buffer(self, device):
        if self._flat is None or self._flat.device != device:
            self._flat = torch.empty(self.numel, dtype=self.dtype, device=device)
        return self._flat

    def pack(self) -> torch.Tensor:
        dev = self.params[0].device
        flat = self._buffer(dev)
        off = 0
        for p in self.params:
            k = p.numel()
            if p.grad is None:
                flat[off:off + k].zero_()
            else:
                flat[off:off + k].copy_(p.grad.reshape(-1))
            off += k
        return flat

    def unpack(self, flat: torch.Tensor) -> None:
        off = 0
        for p in self.params:
            k = p.numel()
            src = flat[off:off + k].view_as(p)
            if p.grad is None:
                p.grad = src.to(p.dtype).clone()
            else:
                p.grad.copy_(src)
            off += k

    def _shared_flat(self) -> Optional[torch.Tensor]:
        """The gradients as one contiguous range of a single buffer, in
        parameter order (the fused backward writes them that way), or None."""
        grads = [p.grad for p in self.params]
        if any(g is None or not g.is_contiguous() or g.dtype != self.dtype for g in grads):
            return None
        base = grads[0]
        ptr = base.data_ptr()
        esize = base.element_size()
        for g in grads:
            if g.untyped_storage().data_ptr() != base.untyped_storage().data_ptr() or \
                    g.data_ptr() != ptr:
                return None
            ptr += g.numel() * esize
        return torch.as_strided(base, (self.numel,), (1,), base.storage_offset())

    def allreduce(self, group=None, async_op: bool = False):
        """Sum (or average) the gradients of all ranks in place."""
        world = dist.get_world_size(group)
        shared = self._shared_flat() if world > 1 else None
        flat = shared if shared is not None else self.pack()
        if world == 1:
            return None
        # NCCL averages inside the collective (no separate scaling kernel);
        # gloo has no AVG, so it sums and scales afterwards
        nccl_avg = self.average and dist.get_backend(group) == "nccl"
        op = dist.ReduceOp.AVG if nccl_avg else dist.ReduceOp.SUM
        work = dist.all_reduce(flat, op=op, group=group, async_op=async_op)

        def finish():
            if work is not None and async_op:
                work.wait()
            if self.average and not nccl_avg:
                flat.div_(world)
            if shared is None:
                self.unpack(flat)

        if async_op:
            return finish
        finish()
        return None


def allreduce_gradients(module: torch.nn.Module, group=None, average: bool = True) -> None:
    """All-reduce every parameter gradient of ``module`` in one flat bucket."""
    GradBucket(module.parameters(), average=average).allreduce(group=group)
