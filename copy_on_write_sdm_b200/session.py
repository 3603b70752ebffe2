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
* ``step_host_pipelined()`` streams host steps through PIPE_DEPTH input and
  output buffers on three streams, so step k+1's inputs cross PCIe while step
  k decodes and step k-1's readouts come back (the decode steps themselves
  stay in order on the compute stream).

The per-step methods issue no autograd-tracked torch operations (only C
calls and host arithmetic), so they skip ``torch.no_grad()``, whose context
costs about 4 us per call -- as much as the rest of a step's host work.

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
from .allocator import POOL_EPOCHS, PackedSDMCopyOnWriteState, new_decode_scratch


def _current_raw_stream(device_index: int) -> int:
    """Handle of torch's current stream on the device (the cheap accessor when present)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


class DecodeSession:
    """Fused decode over ``pools`` with packed input/output buffers.

    Buffer layout (``inputs``, one flat byte buffer, per pool, in order):
    write_indices ``[B,W]``, read_indices ``[B,R]`` (``index_dtype``, int64 by
    default; int32 moves 4 bytes less per index across PCIe in the host-to-host
    steps),
    write_weights ``[B,W]``, read_weights ``[B,R]``, values ``[B,D]``,
    input_gate ``[B]``, forget_log_gate ``[B]`` (activation dtype).  The
    per-pool views are in ``self.views[l]`` (a dict of tensors keyed by the
    ``packed_sdm_cow_step`` argument names); a controller can write its
    routes straight into them.
    """

    FIELDS = ("write_indices", "read_indices", "write_weights", "read_weights", "values", "input_gate",
              "forget_log_gate")

    def __init__(self, pools: Sequence[PackedSDMCopyOnWriteState], *, writes: int, reads: int,
                 act_dtype: torch.dtype = torch.float32, pinned_host: bool = True,
                 index_dtype: torch.dtype = torch.int64) -> None:
        if not 1 <= len(pools) <= _lib.MAX_LAYERS:
            raise ValueError(f"between 1 and {_lib.MAX_LAYERS} pools per session")
        if index_dtype not in (torch.int32, torch.int64):
            raise ValueError("route indices must be int32 or int64")
        p0 = pools[0]
        for p in pools:
            _lib.require_cuda(p.values, "SDM COW state")
            if p.banks != p0.banks or p.width != p0.width or p.values.dtype != p0.values.dtype:
                raise ValueError("session pools must share bank count, width and slab dtype")
        if writes > _lib.MAX_WRITES or reads > _lib.MAX_READS or p0.width % 4 or p0.width > _lib.MAX_WIDTH:
            raise ValueError("route counts or width outside the compiled kernels")
        self.pools = list(pools)
        self._pool_dicts = [p.__dict__ for p in self.pools]
        self.writes, self.reads, self.act_dtype = writes, reads, act_dtype
        self.device = p0.values.device
        B, D = p0.banks, p0.width
        act = torch.tensor([], dtype=act_dtype).element_size()
        shapes = {"write_indices": ((B, writes), index_dtype), "read_indices": ((B, reads), index_dtype),
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
                nbytes = n * (dtype.itemsize if name.endswith("indices") else act)
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
        self._idx_code = _lib.I64 if index_dtype == torch.int64 else _lib.I32
        self._pool_key = None
        self._pool_array = None
        self._scratch = new_decode_scratch(self.device, B * len(pools), len(pools))  # owned by this session
        self._need = B * writes  # first touches one step can make in a pool
        self._proof_steps, self._proof_key = 0, None
        # free counts the decode kernel mirrors to the host (see _prove): the
        # launch counter of this session's scratch, the first launch whose
        # mirror values are trusted, and the page-locked words themselves
        self._issued = 0
        self._mirror_from = 0
        self.snapshot_proofs = 0  # pool proofs renewed from a mirrored count instead of a synchronising read
        self._mirror = torch.zeros(len(pools), dtype=torch.int64, pin_memory=pinned_host)
        self._mirror_np = self._mirror.numpy()
        self._out_bytes = self.host_outputs.numel() * self.host_outputs.element_size()
        self._device_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._lib = _lib.load()
        self._registered: list[torch.Tensor] = []  # pinned host tensors registered with the library

    @staticmethod
    def _views(buf: torch.Tensor, per: dict) -> dict:
        out = {}
        for name, (off, shape, dtype, nbytes) in per.items():
            out[name] = buf[off:off + nbytes].view(dtype).view(shape)
        return out

    def _pools(self):
        key = self._pool_key
        if key is None or key[0] != POOL_EPOCHS[1]:
            versions = tuple(d.get("_tensor_version", 0) for d in self._pool_dicts)
            if key is None or key[1] != versions:
                arr = (_lib.CowPool * len(self.pools))(*[p._pool() for p in self.pools])
                if self._mirror.is_pinned():
                    base = self._mirror.data_ptr()
                    for l in range(len(self.pools)):
                        arr[l].free_mirror = base + 8 * l
                self._pool_array = arr
            self._pool_key = (POOL_EPOCHS[1], versions)
        return self._pool_array

    def _prove(self) -> None:
        """The reference's per-step capacity proof (allocator.py:746-774) for every pool.

        The common case (every pool proven with rows left for this step) is one
        decrement per pool: after a full check the session knows how many steps
        every pool's proof still covers, and keeps that count while no pool was
        assigned to since (the process-wide assignment counter
        ``POOL_EPOCHS[0]`` is unchanged).

        When a proof runs out the reference reads ``free_count`` (a host
        synchronisation).  Here every decode launch writes each pool's settled
        free count, tagged with the launch's epoch, into a page-locked host
        word (``cow_pool.free_mirror``; the epoch counts launches on the
        session's own scan scratch).  A pool whose proof runs out takes
        ``mirror - need x (launches issued after that one)`` as its proof when
        that lower bound covers the step; otherwise, or when a pool was changed
        from outside the session since the mirrored launch, the reference's
        synchronising check runs, so growth happens at exactly the steps where
        the reference grows (the bound never exceeds the true free count).  A
        step run on these pools outside the session goes through
        ``prepare_step_capacity`` (the reference's contract), whose assignment
        makes the session distrust every mirror value written before it."""
        need = self._need
        pools = self._pool_dicts
        epoch = self._issued  # launch epoch of the step being proven
        self._issued += 1
        if self._proof_steps > 0 and self._unchanged_since(self._proof_key):
            self._proof_steps -= 1
            for d in pools:
                d["proven_maximum_additional_allocations"] -= need
            return
        if not self._unchanged_since(self._proof_key):
            self._mirror_from = epoch  # a pool changed outside the session: older mirror values are stale
        bounds = self._mirror_bounds(epoch)
        steps = None
        for l, d in enumerate(pools):
            if d["growth_quantum_rows"]:
                left = d["proven_maximum_additional_allocations"]
                if left >= need and d["capacity_is_proven"]:
                    d["proven_maximum_additional_allocations"] = left - need
                elif bounds is not None and d["capacity_is_proven"] and bounds[l] >= need \
                        and not d["map_table_slots"]:  # hashed pools renew through their table check
                    d["proven_maximum_additional_allocations"] = bounds[l] - need
                    self.snapshot_proofs += 1
                else:
                    self.pools[l].prepare_step_capacity(need)
                left = d["proven_maximum_additional_allocations"] // need if need else 1 << 30
                steps = left if steps is None else min(steps, left)
            elif not d["capacity_is_proven"]:
                raise ValueError("SDM COW capacity has no decode proof")
            else:
                steps = 0  # fixed pools keep the full check (no counter to decrement)
        self._proof_steps = steps or 0
        self._proof_key = self._mutation_key()

    def _mirror_bounds(self, epoch: int):
        """Per-pool lower bounds on the free rows before launch ``epoch``, from the
        mirrored free counts of launches this session may trust; None if none."""
        out = []
        any_valid = False
        for v in self._mirror_np.tolist():
            at, free = (v >> 32) & 0xFFFFFFFF, v & 0xFFFFFFFF
            if v == 0 or at < self._mirror_from or at >= epoch:
                out.append(-1)
                continue
            any_valid = True
            # every launch issued after the mirrored one pops at most `need` rows per pool
            out.append(free - self._need * (epoch - 1 - at))
        return out if any_valid else None

    def _mutation_key(self) -> list:
        """[process-wide assignment count, per-pool assignment counts] now."""
        return [POOL_EPOCHS[0], tuple(d["_mutations"] for d in self._pool_dicts)]

    def _unchanged_since(self, key) -> bool:
        """No pool of this session was assigned to since ``key`` was taken: one
        integer compare when no pool anywhere changed, else the per-pool counts
        (and the key is moved forward so the next check is cheap again)."""
        if key is None:
            return False
        if key[0] == POOL_EPOCHS[0]:
            return True
        if key[1] == tuple(d["_mutations"] for d in self._pool_dicts):
            key[0] = POOL_EPOCHS[0]
            return True
        return False

    def _stream_handle(self) -> int:
        return _current_raw_stream(self._device_index)

    def step(self, *, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """One decode token for every bank of every pool; returns ``outputs`` ``[L, B, D]`` (device)."""
        current = self._stream_handle()
        handle = stream.cuda_stream if stream is not None else current
        self._prove()
        _lib.check(self._lib.cow_decode_step(self._pools(), self._steps, len(self.pools), self.writes, self.reads,
                                             self._idx_code, self._act_code, self._scratch.data_ptr(),
                                             self._scratch.numel(), handle), "cow_decode_step")
        return self.outputs

    # Buffer pairs the host-to-host pipelines rotate through: a step's input
    # copy waits only for the decode that read its buffer PIPE_DEPTH steps
    # earlier, so copies of several neighbouring steps can be in flight.
    PIPE_DEPTH = 4

    def _pipeline(self):
        if self._pipe is None:
            n = self.PIPE_DEPTH
            inputs = [self.inputs] + [torch.empty_like(self.inputs) for _ in range(n - 1)]
            outputs = [self.outputs] + [torch.empty_like(self.outputs) for _ in range(n - 1)]
            steps = [self._steps]
            for b in range(1, n):
                views = [self._views(inputs[b], per) for per in self._offsets]
                steps.append((_lib.CowStep * len(self.pools))(*[
                    _lib.CowStep(v["write_indices"].data_ptr(), v["write_weights"].data_ptr(),
                                 v["values"].data_ptr(), v["input_gate"].data_ptr(), v["input_gate"].data_ptr(),
                                 v["forget_log_gate"].data_ptr(), v["read_indices"].data_ptr(),
                                 v["read_weights"].data_ptr(), outputs[b][l].data_ptr(), None)
                    for l, v in enumerate(views)]))
            pinned = self.host_outputs.is_pinned()
            h2d, d2h = torch.cuda.Stream(self.device), torch.cuda.Stream(self.device)
            events = [[torch.cuda.Event() for _ in range(3)] for _ in range(n)]
            for group in events:  # materialise the handles; a recorded-then-idle event never blocks
                for ev in group:
                    ev.record(h2d)
            torch.cuda.synchronize(self.device)
            host_outputs = [self.host_outputs] + [torch.empty_like(self.host_outputs, pin_memory=pinned)
                                                  for _ in range(n - 1)]
            # one descriptor per buffer pair: every argument of the overlapped step
            # but the host input bytes and the compute stream
            descs = tuple(_lib.CowHostPipeline(
                None, ctypes.cast(steps[b], ctypes.POINTER(_lib.CowStep)), len(self.pools), self.writes, self.reads,
                self._idx_code, self._act_code, 0, self._scratch.data_ptr(), self._scratch.numel(), inputs[b].data_ptr(),
                self.step_bytes, host_outputs[b].data_ptr(), outputs[b].data_ptr(), self._out_bytes,
                h2d.cuda_stream, d2h.cuda_stream, events[b][0].cuda_event, events[b][1].cuda_event,
                events[b][2].cuda_event) for b in range(n))
            for t in host_outputs:
                self._register(t)
            self._pipe = {
                "inputs": inputs, "outputs": outputs, "steps": steps, "host_outputs": host_outputs,
                "h2d": h2d, "d2h": d2h, "events": events, "k": 0, "descs": descs, "depth": n,
                "desc_ptrs": tuple(ctypes.addressof(d) for d in descs), "desc_pools": None,
            }
        return self._pipe

    def step_host_pipelined(self, host_step: torch.Tensor) -> tuple[torch.Tensor, torch.cuda.Event]:
        """Host-to-host step overlapped with its neighbours (``cow_decode_step_host_piped``).

        ``host_step`` holds the step's pinned input bytes (``inputs`` layout).
        Returns the pinned host buffer that will hold this step's readouts
        ``[L, B, D]`` and the event that marks their arrival; the buffer is
        reused PIPE_DEPTH steps later.  Steps decode strictly in call order on the
        current stream; the copies run on two side streams.
        """
        if host_step.nbytes != self.step_bytes or host_step.dtype is not torch.uint8 \
                or host_step.is_cuda or not host_step.is_contiguous():
            raise ValueError(f"host step must be {self.step_bytes} contiguous uint8 bytes on the host")
        pipe = self._pipe if self._pipe is not None else self._pipeline()
        b = pipe["k"] % pipe["depth"]
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

    def _register(self, t: torch.Tensor) -> None:
        if t.is_pinned() and self._lib.cow_register_host_range(t.data_ptr(), t.numel() * t.element_size()) == 0:
            self._registered.append(t)  # held until close(): the library keeps its address

    def register_host_steps(self, host_steps: torch.Tensor) -> None:
        """Register a pinned buffer of host steps (e.g. ``[K, step_bytes]`` uint8) for
        ``step_host_mapped``: steps inside it skip the per-call pinned-memory query.
        The session holds the tensor until ``close()``."""
        if not host_steps.is_pinned() or not host_steps.is_contiguous():
            raise ValueError("host steps must be a contiguous pinned tensor")
        _lib.check(self._lib.cow_register_host_range(host_steps.data_ptr(),
                                                     host_steps.numel() * host_steps.element_size()),
                   "cow_register_host_range")
        self._registered.append(host_steps)

    def close(self) -> None:
        """Forget the host ranges this session registered (idempotent)."""
        lib = getattr(self, "_lib", None)
        for t in getattr(self, "_registered", ()):
            if lib is not None:
                lib.cow_unregister_host_range(t.data_ptr())
        self._registered = []

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def step_host_mapped(self, host_step: torch.Tensor) -> tuple[torch.Tensor, torch.cuda.Event]:
        """Host-to-host step with no copy calls (``cow_decode_step_host_mapped``).

        The decode kernel reads ``host_step`` (pinned bytes in the ``inputs``
        layout) over PCIe and writes the readouts straight into a pinned host
        buffer: one kernel launch per token.  Returns that buffer ``[L, B, D]``
        and the event that marks the readouts' arrival; the buffer is reused
        PIPE_DEPTH steps later, and ``host_step`` must stay untouched until the event
        has completed.  Steps decode in call order on the current stream.
        """
        if host_step.nbytes != self.step_bytes or host_step.dtype is not torch.uint8 \
                or host_step.is_cuda or not host_step.is_contiguous():
            raise ValueError(f"host step must be {self.step_bytes} contiguous uint8 bytes on the host")
        ptr = host_step.data_ptr()
        pipe = self._pipe if self._pipe is not None else self._pipeline()
        b = pipe["k"] % pipe["depth"]
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

    def step_host(self, host_step: torch.Tensor | None = None) -> torch.Tensor:
        """Host-to-host step: copy ``host_step`` (pinned bytes in the ``inputs`` layout,
        default ``host_inputs``) to the device, decode, copy the readouts back into
        ``host_outputs`` (asynchronously on the current stream) and return it."""
        src = self.host_inputs if host_step is None else host_step
        if src.numel() != self.step_bytes or src.dtype != torch.uint8 or src.is_cuda \
                or not src.is_contiguous():
            raise ValueError(f"host step must be {self.step_bytes} contiguous uint8 bytes on the host")
        self._prove()
        out = self.host_outputs
        _lib.check(self._lib.cow_decode_step_host(
            self._pools(), self._steps, len(self.pools), self.writes, self.reads, self._idx_code, self._act_code,
            self._scratch.data_ptr(), self._scratch.numel(), self.inputs.data_ptr(), src.data_ptr(), self.step_bytes,
            out.data_ptr(), self.outputs.data_ptr(), self._out_bytes, self._stream_handle()),
            "cow_decode_step_host")
        return out
