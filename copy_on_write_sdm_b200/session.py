"""Low-overhead decode runtime over a fixed set of packed pools.

``packed_sdm_cow_step_layers`` validates and re-wraps every tensor on each
call, which costs tens of microseconds of host time -- more than the decode
launch itself at serving batch sizes.  ``DecodeSession`` does that work once:

* it owns one contiguous device buffer holding every pool's step inputs
  (write/read indices, weights, values, gates) and one output buffer, so a
  step's inputs arrive with ONE host->device copy and its readouts leave with
  ONE device->host copy;
* it keeps the C-ABI pool and step descriptors prebuilt, rebuilding the pool
  descriptors only when a pool's tensors were replaced (growth, trim,
  admission);
* ``step()`` runs the reference's per-step capacity proof
  (``prepare_step_capacity``, allocator.py:746-774) for every pool, then one
  fused ``cow_decode_step`` launch for all pools.

Semantics per pool are exactly ``packed_sdm_cow_step`` with
``validate_routes=False, collect_diagnostics=False`` (the decode path of
inference.py:538-566); every pool must have the same bank count, width and
route counts.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib
from .allocator import PackedSDMCopyOnWriteState, decode_scratch


class DecodeSession:
    """Fused decode over ``pools`` with packed input/output buffers.

    Buffer layout (``inputs``, one flat byte buffer, per pool, in order):
    write_indices ``[B,W]`` int64, read_indices ``[B,R]`` int64,
    write_weights ``[B,W]``, read_weights ``[B,R]``, values ``[B,D]``,
    input_gate ``[B]``, forget_log_gate ``[B]`` (activation dtype).  The
    per-pool views are in ``self.views[l]`` (a dict of tensors keyed by the
    ``packed_sdm_cow_step`` argument names); a controller can write its
    routes straight into them.
    """

    FIELDS = ("write_indices", "read_indices", "write_weights", "read_weights", "values", "input_gate",
              "forget_log_gate")

    def __init__(self, pools: Sequence[PackedSDMCopyOnWriteState], *, writes: int, reads: int,
                 act_dtype: torch.dtype = torch.float32, pinned_host: bool = True) -> None:
        if not 1 <= len(pools) <= _lib.MAX_LAYERS:
            raise ValueError(f"between 1 and {_lib.MAX_LAYERS} pools per session")
        p0 = pools[0]
        for p in pools:
            _lib.require_cuda(p.values, "SDM COW state")
            if p.banks != p0.banks or p.width != p0.width or p.values.dtype != p0.values.dtype:
                raise ValueError("session pools must share bank count, width and slab dtype")
        if writes > _lib.MAX_WRITES or reads > _lib.MAX_READS or p0.width % 4 or p0.width > _lib.MAX_WIDTH:
            raise ValueError("route counts or width outside the compiled kernels")
        self.pools = list(pools)
        self.writes, self.reads, self.act_dtype = writes, reads, act_dtype
        self.device = p0.values.device
        B, D = p0.banks, p0.width
        act = torch.tensor([], dtype=act_dtype).element_size()
        shapes = {"write_indices": ((B, writes), torch.int64), "read_indices": ((B, reads), torch.int64),
                  "write_weights": ((B, writes), act_dtype), "read_weights": ((B, reads), act_dtype),
                  "values": ((B, D), act_dtype), "input_gate": ((B,), act_dtype),
                  "forget_log_gate": ((B,), act_dtype)}
        # 16-byte aligned sub-buffers inside one allocation
        offsets, off = [], 0
        for _ in pools:
            per = {}
            for name in self.FIELDS:
                shape, dtype = shapes[name]
                n = 1
                for s in shape:
                    n *= s
                nbytes = n * (8 if dtype == torch.int64 else act)
                per[name] = (off, shape, dtype, nbytes)
                off += (nbytes + 15) // 16 * 16
            offsets.append(per)
        self.step_bytes = off
        self.inputs = torch.empty(off, dtype=torch.uint8, device=self.device)
        self.host_inputs = torch.empty(off, dtype=torch.uint8, pin_memory=pinned_host)
        self.outputs = torch.empty(len(pools), B, D, dtype=act_dtype, device=self.device)
        self.host_outputs = torch.empty(len(pools), B, D, dtype=act_dtype, pin_memory=pinned_host)
        self.views = [self._views(self.inputs, per) for per in offsets]
        self.host_views = [self._views(self.host_inputs, per) for per in offsets]
        self._steps = (_lib.CowStep * len(pools))(*[
            _lib.CowStep(v["write_indices"].data_ptr(), v["write_weights"].data_ptr(), v["values"].data_ptr(),
                         v["input_gate"].data_ptr(), v["input_gate"].data_ptr(), v["forget_log_gate"].data_ptr(),
                         v["read_indices"].data_ptr(), v["read_weights"].data_ptr(), self.outputs[l].data_ptr(),
                         None)
            for l, v in enumerate(self.views)])
        self._act_code = _lib.dtype_code(act_dtype)
        self._pool_key = None
        self._pool_array = None
        self._scratch = decode_scratch(self.device, B * len(pools), len(pools))
        self._lib = _lib.load()

    @staticmethod
    def _views(buf: torch.Tensor, per: dict) -> dict:
        out = {}
        for name, (off, shape, dtype, nbytes) in per.items():
            out[name] = buf[off:off + nbytes].view(dtype).view(shape)
        return out

    def _pools(self):
        key = tuple((p.values.data_ptr(), p.logical_to_physical.data_ptr(), p.free_rows.data_ptr(),
                     p.template_indices.data_ptr(), p.capacity_rows, p.banks) for p in self.pools)
        if key != self._pool_key:
            self._pool_array = (_lib.CowPool * len(self.pools))(*[p._pool() for p in self.pools])
            self._pool_key = key
        return self._pool_array

    @torch.no_grad()
    def step(self, *, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """One decode token for every bank of every pool; returns ``outputs`` ``[L, B, D]`` (device)."""
        for p in self.pools:
            if p.growth_quantum_rows:
                p.prepare_step_capacity(p.banks * self.writes)
            elif not p.capacity_is_proven:
                raise ValueError("SDM COW capacity has no decode proof")
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(self._lib.cow_decode_step(self._pools(), self._steps, len(self.pools), self.writes, self.reads,
                                             _lib.I64, self._act_code, self._scratch.data_ptr(),
                                             self._scratch.numel(), s.cuda_stream), "cow_decode_step")
        return self.outputs

    @torch.no_grad()
    def step_host(self, host_step: torch.Tensor | None = None) -> torch.Tensor:
        """Host-to-host step: copy ``host_step`` (pinned bytes in the ``inputs`` layout,
        default ``host_inputs``) to the device, decode, copy the readouts back into
        ``host_outputs`` (asynchronously on the current stream) and return it."""
        src = self.host_inputs if host_step is None else host_step
        self.inputs.copy_(src, non_blocking=True)
        self.step()
        self.host_outputs.copy_(self.outputs, non_blocking=True)
        return self.host_outputs
