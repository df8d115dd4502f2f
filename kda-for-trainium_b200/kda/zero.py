"""ZeRO-1 AdamW: the optimizer step that follows the adamw operator in data-
parallel training, sharded over the ranks of one node.

Every rank holds the full flat fp32 parameter buffer (replicated, as the
forward/backward needs it) and a full flat gradient buffer (its local
gradients); each rank owns the AdamW moments of one contiguous shard.  One
step is: average the gradients of its shard over all ranks (reduce-scatter),
AdamW on that shard, and give every rank the updated shard (all-gather).

``fused=True`` (the default on GPUs) runs the whole step as ONE kernel per rank
(``kda_zero1_adamw_f32``): it reads the shard of every rank's gradient buffer
over NVLink (CUDA IPC mappings), updates the shard, and stores the new
parameters into every rank's buffer.  The host orders it with two stream-
ordered collectives (a one-element all-reduce before, so every rank's
gradients are complete, and after, so every peer store has landed and nobody
overwrites a gradient buffer another rank is still reading).  ``fused=False``
is the collective baseline: reduce-scatter, multi-tensor AdamW, all-gather.

The reference's adamw forward is one step of this optimizer with lr 1e-3,
betas (0.9, 0.999), eps 1e-8, weight decay 1e-2 at step 1
(``workspaces/adamw/runs/adamw_v1.py:5-11``, ``prompts/_gen_prompts.py:227-228``);
those are the defaults here.
"""

from __future__ import annotations

import ctypes as C
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib, ops


def shard_bounds(numel: int, world: int):
    """(padded length, shard length): the flat buffers are padded so every
    rank's shard has the same length, a multiple of 4 elements (16 bytes)."""
    if numel < 0 or world < 1:
        raise ValueError(f"bad numel {numel} / world {world}")
    unit = 4 * world
    padded = max(unit, -(-numel // unit) * unit)
    return padded, padded // world


class Zero1AdamW:
    """ZeRO-1 AdamW over a flat fp32 parameter buffer of ``numel`` elements.

    ``param`` and ``grad`` are the padded flat buffers (write gradients into
    ``grad[:numel]``; the padding stays zero).  ``update`` replaces the
    per-shard AdamW of the collective path (a hook for tests on CPU ranks,
    where no CUDA kernel can run); the fused path has no such hook.
    """

    def __init__(self, numel: int, *, device=None, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, fused: Optional[bool] = None, group=None,
                 update: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.numel = int(numel)
        self.padded, self.shard_len = shard_bounds(self.numel, self.world)
        self.off = self.rank * self.shard_len
        self.lr, self.betas, self.eps, self.weight_decay = float(lr), tuple(map(float, betas)), float(eps), \
            float(weight_decay)
        self.step_count = 0
        on_gpu = self.device.type == "cuda"
        self.fused = (on_gpu and self.world > 1) if fused is None else bool(fused)
        if self.fused and (not on_gpu or update is not None):
            raise ValueError("the fused ZeRO-1 step runs on CUDA devices with the library's kernel")
        if self.fused and self.world > 8:
            raise ValueError("the fused ZeRO-1 step supports up to 8 ranks (one node)")
        self.update = update
        self.param = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        self.m = torch.zeros(self.shard_len, dtype=torch.float32, device=self.device)
        self.v = torch.zeros(self.shard_len, dtype=torch.float32, device=self.device)
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._peers = None
        if self.fused:
            self._map_peers()

    @classmethod
    def for_tensors(cls, tensors, **kw):
        """A ZeRO-1 optimizer over a list of fp32 parameter tensors (a model's
        parameters, identical on every rank): their values are copied into the
        flat buffer, and (optimizer, param_views, grad_views) is returned --
        views shaped like the tensors, into ``param`` and ``grad``, for the model
        to compute with and to write its gradients into."""
        tensors = list(tensors)
        numel = sum(t.numel() for t in tensors)
        dev = tensors[0].device if tensors else None
        opt = cls(numel, device=kw.pop("device", dev), **kw)
        pv, gv, off = [], [], 0
        for t in tensors:
            n = t.numel()
            p = opt.param[off:off + n].view(t.shape)
            p.copy_(t.detach())
            pv.append(p)
            gv.append(opt.grad[off:off + n].view(t.shape))
            off += n
        return opt, pv, gv

    # ------------------------------------------------------------ peer memory
    def _map_peers(self):
        if self.world == 1:  # nothing to map: the step reads and writes this rank's buffers
            self._peers = ((C.c_void_p * 1)(self.param.data_ptr()), (C.c_void_p * 1)(self.grad.data_ptr()), [])
            return
        lib = _lib.lib()
        hsize = int(_lib._attach(lib, "kda_ipc_handle_size")())
        mine = []
        for buf in (self.param, self.grad):
            h = (C.c_ubyte * hsize)()
            off = C.c_int64(0)
            with torch.cuda.device(self.device):
                _lib.call("kda_ipc_export", C.c_void_p(buf.data_ptr()), h, C.byref(off))
            mine.append((bytes(h), off.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=self.group)
        params, grads, opened = [], [], []
        for r in range(self.world):
            if r == self.rank:
                params.append(self.param.data_ptr())
                grads.append(self.grad.data_ptr())
                continue
            ptrs = []
            for hb, off in allh[r]:
                p = C.c_void_p(0)
                h = (C.c_ubyte * hsize).from_buffer_copy(hb)
                with torch.cuda.device(self.device):
                    _lib.call("kda_ipc_open", h, C.c_int64(off), C.byref(p))
                ptrs.append(p.value)
                opened.append((p.value, off))
            params.append(ptrs[0])
            grads.append(ptrs[1])
        self._peers = ((C.c_void_p * self.world)(*params), (C.c_void_p * self.world)(*grads), opened)

    def close(self):
        """Unmap the peers' buffers (after a final barrier: no peer still
        stores into this rank's parameters)."""
        if self._peers is None:
            return
        self._barrier()
        torch.cuda.synchronize(self.device)
        for p, off in self._peers[2]:
            with torch.cuda.device(self.device):
                _lib.call("kda_ipc_close", C.c_void_p(p), C.c_int64(off))
        self._peers = None

    def _barrier(self):
        # stream-ordered: completes only after every rank's earlier work on its stream
        if self.world > 1:
            dist.all_reduce(self._flag, group=self.group)

    # -------------------------------------------------------------------- step
    def step(self):
        """One optimizer step from the gradients in ``grad`` (all ranks)."""
        self.step_count += 1
        b1, b2 = self.betas
        if self.fused:
            self._barrier()
            with torch.cuda.device(self.device):
                _lib.call("kda_zero1_adamw_f32", self._peers[1], self._peers[0], self.world, self.rank,
                          self.off, self.shard_len, C.c_void_p(self.m.data_ptr()), C.c_void_p(self.v.data_ptr()),
                          self.lr, b1, b2, self.eps, self.weight_decay, self.step_count,
                          C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
            self._barrier()
            return
        gshard = self._reduce_scatter()
        pshard = self.param[self.off:self.off + self.shard_len]
        if self.update is not None:
            self.update(pshard, gshard, self.m, self.v, lr=self.lr, betas=self.betas, eps=self.eps,
                        weight_decay=self.weight_decay, step=self.step_count)
        else:
            ops.adamw_multi([pshard], [gshard], [self.m], [self.v], lr=self.lr, betas=self.betas, eps=self.eps,
                            weight_decay=self.weight_decay, step=self.step_count)
        self._all_gather(pshard)

    def _reduce_scatter(self):
        out = torch.empty(self.shard_len, dtype=torch.float32, device=self.device)
        if self.world == 1:
            out.copy_(self.grad)
        elif dist.get_backend(self.group) == "nccl":
            dist.reduce_scatter_tensor(out, self.grad, op=dist.ReduceOp.SUM, group=self.group)
        else:  # gloo has no reduce-scatter: all-reduce a copy, keep this rank's shard
            full = self.grad.clone()
            dist.all_reduce(full, group=self.group)
            out.copy_(full[self.off:self.off + self.shard_len])
        return out.mul_(1.0 / self.world)

    def _all_gather(self, pshard):
        if self.world == 1:
            return
        src = pshard.clone()
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self.param, src, group=self.group)
        else:
            parts = list(self.param.view(self.world, self.shard_len).unbind(0))
            dist.all_gather(parts, src, group=self.group)
