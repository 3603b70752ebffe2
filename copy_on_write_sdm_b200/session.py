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
  fused ``cow_decode_step`` launch for all pools;
* ``step_host_pipelined()`` streams host steps through two input and two
  output buffers on three streams, so step k+1's inputs cross PCIe while step
  k decodes and step k-1's readouts come back (the decode steps themselves
  stay in order on the compute stream).

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
from .allocator import PackedSDMCopyOnWriteState, new_decode_scratch


def _current_raw_stream(device_index: int) -> int:
    """Handle of torch's current stream on the device (the cheap accessor when present)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


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
        self._offsets = offsets
        self._pipe = None
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
        self._scratch = new_decode_scratch(self.device, B * len(pools), len(pools))  # owned by this session
        self._need = B * writes  # first touches one step can make in a pool
        self._proof_steps, self._proof_key = 0, None
        # free-count snapshots copied to the host without a synchronisation
        # (see _prove): the issued-step counter, the pending snapshot and its
        # pinned landing buffer
        self._issued = 0
        self._snap = None
        self._snapshots = True  # off for good once a step decodes on another stream than the current one
        self.snapshot_proofs = 0  # pool proofs renewed from a snapshot instead of a synchronising read
        self._snap_host = torch.empty(len(pools), dtype=torch.int32, pin_memory=pinned_host)
        self._out_bytes = self.host_outputs.numel() * self.host_outputs.element_size()
        self._device_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._lib = _lib.load()

    @staticmethod
    def _views(buf: torch.Tensor, per: dict) -> dict:
        out = {}
        for name, (off, shape, dtype, nbytes) in per.items():
            out[name] = buf[off:off + nbytes].view(dtype).view(shape)
        return out

    def _pools(self):
        key = tuple(p.__dict__.get("_tensor_version", 0) for p in self.pools)
        if key != self._pool_key:
            self._pool_array = (_lib.CowPool * len(self.pools))(*[p._pool() for p in self.pools])
            self._pool_key = key
        return self._pool_array

    def _prove(self, on_current: bool = True) -> None:
        """The reference's per-step capacity proof (allocator.py:746-774) for every pool.

        The common case (every pool proven with rows left for this step) is one
        decrement per pool: after a full check the session knows how many steps
        every pool's proof still covers, and keeps that count while no pool was
        assigned to since (its ``_mutations`` counter is unchanged).

        When a proof runs out the reference reads ``free_count`` (a host
        synchronisation).  Two steps before that, the session copies every
        pool's free count to pinned host memory in the background; a pool whose
        proof runs out then takes ``snapshot - need x (steps issued after it)``
        as its proof when that lower bound covers the step.  Otherwise, or when
        the snapshot has not landed or a pool changed since, the reference's
        synchronising check runs, so growth happens at exactly the steps where
        the reference grows (the bound never exceeds the true free count).
        Snapshots are taken and used only while every step decodes on the current
        stream, which orders them with the decodes they must follow.  A step run on
        these pools outside the session goes through ``prepare_step_capacity`` (the
        reference's contract), whose assignment invalidates a pending snapshot."""
        need = self._need
        pools = self.pools
        self._issued += 1
        if not on_current:
            self._snapshots, self._snap = False, None
        if self._proof_steps > 0 and self._proof_key == tuple(p.__dict__["_mutations"] for p in pools):
            self._proof_steps -= 1
            for p in pools:
                d = p.__dict__
                d["proven_maximum_additional_allocations"] -= need
            if self._proof_steps <= 2 and self._snap is None and self._snapshots:
                self._snapshot()
            return
        snap = self._snap_bounds()
        steps = None
        for l, p in enumerate(pools):
            d = p.__dict__
            if d["growth_quantum_rows"]:
                left = d["proven_maximum_additional_allocations"]
                if left >= need and d["capacity_is_proven"]:
                    d["proven_maximum_additional_allocations"] = left - need
                elif snap is not None and d["capacity_is_proven"] and snap[l] >= need:
                    d["proven_maximum_additional_allocations"] = snap[l] - need
                    self.snapshot_proofs += 1
                else:
                    p.prepare_step_capacity(need)
                left = d["proven_maximum_additional_allocations"] // need if need else 1 << 30
                steps = left if steps is None else min(steps, left)
            elif not d["capacity_is_proven"]:
                raise ValueError("SDM COW capacity has no decode proof")
            else:
                steps = 0  # fixed pools keep the full check (no counter to decrement)
        self._proof_steps = steps or 0
        self._proof_key = tuple(p.__dict__["_mutations"] for p in pools)

    def _snapshot(self) -> None:
        """Queue a copy of every pool's free count (after the steps issued so far) to
        pinned host memory on the current stream (not while it is being captured)."""
        if torch.cuda.is_current_stream_capturing():
            return
        counts = torch.cat([p.free_count.reshape(1) for p in self.pools])
        self._snap_host.copy_(counts, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._snap = (ev, self._issued - 1, tuple(p.__dict__["_mutations"] for p in self.pools))

    def _snap_bounds(self):
        """Per-pool lower bounds on the free rows before the step being issued, from a
        landed snapshot taken since the pools last changed; None otherwise."""
        snap, self._snap = self._snap, None
        if snap is None:
            return None
        ev, at, key = snap
        if key != tuple(p.__dict__["_mutations"] for p in self.pools) or torch.cuda.is_current_stream_capturing() \
                or not ev.query():
            return None
        # every step issued after the snapshot pops at most `need` rows per pool
        charged = self._need * (self._issued - 1 - at)
        return [int(c) - charged for c in self._snap_host.tolist()]

    def _stream_handle(self) -> int:
        return _current_raw_stream(self._device_index)

    @torch.no_grad()
    def step(self, *, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """One decode token for every bank of every pool; returns ``outputs`` ``[L, B, D]`` (device)."""
        current = self._stream_handle()
        handle = stream.cuda_stream if stream is not None else current
        self._prove(on_current=handle == current)
        _lib.check(self._lib.cow_decode_step(self._pools(), self._steps, len(self.pools), self.writes, self.reads,
                                             _lib.I64, self._act_code, self._scratch.data_ptr(),
                                             self._scratch.numel(), handle), "cow_decode_step")
        return self.outputs

    def _pipeline(self):
        if self._pipe is None:
            alt = torch.empty_like(self.inputs)
            views = [self._views(alt, per) for per in self._offsets]
            out_alt = torch.empty_like(self.outputs)
            steps_alt = (_lib.CowStep * len(self.pools))(*[
                _lib.CowStep(v["write_indices"].data_ptr(), v["write_weights"].data_ptr(), v["values"].data_ptr(),
                             v["input_gate"].data_ptr(), v["input_gate"].data_ptr(), v["forget_log_gate"].data_ptr(),
                             v["read_indices"].data_ptr(), v["read_weights"].data_ptr(), out_alt[l].data_ptr(), None)
                for l, v in enumerate(views)])
            pinned = self.host_outputs.is_pinned()
            h2d, d2h = torch.cuda.Stream(self.device), torch.cuda.Stream(self.device)
            events = [[torch.cuda.Event() for _ in range(3)] for _ in range(2)]
            for pair in events:  # materialise the handles; a recorded-then-idle event never blocks
                for ev in pair:
                    ev.record(h2d)
            torch.cuda.synchronize(self.device)
            host_outputs = (self.host_outputs, torch.empty_like(self.host_outputs, pin_memory=pinned))
            inputs, outputs, steps = (self.inputs, alt), (self.outputs, out_alt), (self._steps, steps_alt)
            # one descriptor per buffer pair: every argument of the overlapped step
            # but the host input bytes and the compute stream
            descs = tuple(_lib.CowHostPipeline(
                None, ctypes.cast(steps[b], ctypes.POINTER(_lib.CowStep)), len(self.pools), self.writes, self.reads,
                _lib.I64, self._act_code, 0, self._scratch.data_ptr(), self._scratch.numel(), inputs[b].data_ptr(),
                self.step_bytes, host_outputs[b].data_ptr(), outputs[b].data_ptr(), self._out_bytes,
                h2d.cuda_stream, d2h.cuda_stream, events[b][0].cuda_event, events[b][1].cuda_event,
                events[b][2].cuda_event) for b in range(2))
            self._pipe = {
                "inputs": inputs, "outputs": outputs, "steps": steps, "host_outputs": host_outputs,
                "h2d": h2d, "d2h": d2h, "events": events, "k": 0, "descs": descs,
                "desc_ptrs": tuple(ctypes.addressof(d) for d in descs), "desc_pools": None,
            }
        return self._pipe

    @torch.no_grad()
    def step_host_pipelined(self, host_step: torch.Tensor) -> tuple[torch.Tensor, torch.cuda.Event]:
        """Host-to-host step overlapped with its neighbours (``cow_decode_step_host_piped``).

        ``host_step`` holds the step's pinned input bytes (``inputs`` layout).
        Returns the pinned host buffer that will hold this step's readouts
        ``[L, B, D]`` and the event that marks their arrival; the buffer is
        reused two steps later.  Steps decode strictly in call order on the
        current stream; the copies run on two side streams.
        """
        if host_step.numel() != self.step_bytes or host_step.dtype != torch.uint8 \
                or host_step.device.type != "cpu" or not host_step.is_contiguous():
            raise ValueError(f"host step must be {self.step_bytes} contiguous uint8 bytes on the host")
        pipe = self._pipe if self._pipe is not None else self._pipeline()
        b = pipe["k"] & 1
        pipe["k"] += 1
        self._prove()
        pools = self._pools()
        if pipe["desc_pools"] is not pools:  # a pool's tensors were replaced: new pool array
            for d in pipe["descs"]:
                d.pools = ctypes.cast(pools, ctypes.POINTER(_lib.CowPool))
            pipe["desc_pools"] = pools
        rc = self._lib.cow_decode_step_host_piped(pipe["desc_ptrs"][b], host_step.data_ptr(), self._stream_handle())
        if rc:
            _lib.check(rc, "cow_decode_step_host_piped")
        return pipe["host_outputs"][b], pipe["events"][b][2]

    @torch.no_grad()
    def step_host_mapped(self, host_step: torch.Tensor) -> tuple[torch.Tensor, torch.cuda.Event]:
        """Host-to-host step with no copy calls (``cow_decode_step_host_mapped``).

        The decode kernel reads ``host_step`` (pinned bytes in the ``inputs``
        layout) over PCIe and writes the readouts straight into a pinned host
        buffer: one kernel launch per token.  Returns that buffer ``[L, B, D]``
        and the event that marks the readouts' arrival; the buffer is reused
        two steps later, and ``host_step`` must stay untouched until the event
        has completed.  Steps decode in call order on the current stream.
        """
        if host_step.numel() != self.step_bytes or host_step.dtype != torch.uint8 \
                or host_step.device.type != "cpu" or not host_step.is_contiguous():
            raise ValueError(f"host step must be {self.step_bytes} contiguous uint8 bytes on the host")
        ptr = host_step.data_ptr()
        pipe = self._pipe if self._pipe is not None else self._pipeline()
        b = pipe["k"] & 1
        pipe["k"] += 1
        self._prove()
        pools = self._pools()
        if pipe["desc_pools"] is not pools:
            for d in pipe["descs"]:
                d.pools = ctypes.cast(pools, ctypes.POINTER(_lib.CowPool))
            pipe["desc_pools"] = pools
        out = pipe["host_outputs"][b]
        rc = self._lib.cow_decode_step_host_mapped(pipe["desc_ptrs"][b], ptr, out.data_ptr(), self._stream_handle())
        if rc:
            if rc == _lib.ERR_INVALID:
                raise ValueError("mapped host steps must live in pinned (page-locked) host memory")
            _lib.check(rc, "cow_decode_step_host_mapped")
        return out, pipe["events"][b][2]

    @torch.no_grad()
    def step_host(self, host_step: torch.Tensor | None = None) -> torch.Tensor:
        """Host-to-host step: copy ``host_step`` (pinned bytes in the ``inputs`` layout,
        default ``host_inputs``) to the device, decode, copy the readouts back into
        ``host_outputs`` (asynchronously on the current stream) and return it."""
        src = self.host_inputs if host_step is None else host_step
        if src.numel() != self.step_bytes or src.dtype != torch.uint8 or src.device.type != "cpu" \
                or not src.is_contiguous():
            raise ValueError(f"host step must be {self.step_bytes} contiguous uint8 bytes on the host")
        self._prove()
        out = self.host_outputs
        _lib.check(self._lib.cow_decode_step_host(
            self._pools(), self._steps, len(self.pools), self.writes, self.reads, _lib.I64, self._act_code,
            self._scratch.data_ptr(), self._scratch.numel(), self.inputs.data_ptr(), src.data_ptr(), self.step_bytes,
            out.data_ptr(), self.outputs.data_ptr(), self._out_bytes, self._stream_handle()),
            "cow_decode_step_host")
        return out
