"""Packed-SDM decode benchmark (BASELINE metric: decode tokens/s at batch 64 per GPU).

Workload (configuration 3, the synthetic random-route serving screen): 7
independent SDM pools (layers), N=256 slots, D=128, H=1, top-16 reads / top-4
writes, uniform seeded routes, batch 64 requests per GPU, prefix 2,048 tokens
(sparse prefill handoff), then decode with a four-step growth quantum
(``max(16, 64*4*4) = 1,024`` rows).  One *step* = one decode token for every
request through all 7 pools = one fused ``cow_decode_step`` launch.

Reported numbers (one JSON line from rank 0):

* ``value``: device throughput, inputs resident in HBM.  The K timed steps
  are ONE CUDA graph between one device event pair; step i runs on replica
  i mod REPLICAS of the pools (independent copies of this GPU's state), so
  more than twice the L2 is moved between two visits of a replica and every
  step starts cold without a flush.  ``flushed_event_timed`` is the same K
  steps on the pools themselves as K x (256 MiB L2 flush, event, the fused
  launch, event) in one graph; ``single_launch`` is one step launched and
  timed alone (each interval then also holds the host's submission latency).
* ``e2e``: the same metric through the public runtime API with host buffers:
  every step copies its packed routes from pinned host memory (one copy), runs
  the capacity proof and one fused launch, and reads the readouts back to the
  host, through ``DecodeSession.step_host_pipelined`` (the copies of
  neighbouring steps overlap the decode); ``e2e.serial`` is the
  one-step-at-a-time ``DecodeSession.step_host``.
* ``roofline``: algorithmic bytes per launch / mean launch time vs the
  measured HBM copy bandwidth.
* ``dense_control``: the dense-table control kernel timed the same way, and
  the packed path's latency overhead against it.
* ``cpu_baseline``: the CPU restatement of the reference's deterministic
  path, timed on a bounded sample on this host.

Multi-GPU: one process per GPU (torchrun); each rank owns its own 64
requests (weak scaling, no collective on the data path); time is the max over
ranks.  ``--impl reference`` times the reference's CPU algorithm instead.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "packed-SDM decode tokens/s at batch 64, 1/2/4/8 B200; % of HBM roofline"
LAYERS, SLOTS, WIDTH, HEADS, READS, WRITES = 7, 256, 128, 1, 16, 4
BATCH, PREFIX, QUANTUM_STEPS = 64, 2048, 4
L2_FLUSH_BYTES = 256 << 20
REPLICAS = 48  # independent copies of the pools the timed trace cycles through
E2E_WARMUP = 64  # untimed host-to-host steps before each end-to-end leg
# DRAM traffic per launch of the dominant kernel from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum); the capture commands and
# figures are in profiles/.
TRAFFIC_SCREEN = {"bytes_per_launch": 5_364_224,
                  "source": "ncu, cow_decode_split_kernel (read rows in registers), bench.py --steps 4 --warmup 3 "
                            "--no-legs, two flushed launches: dram__bytes_read.sum 5.36 MB + dram__bytes_write.sum "
                            "0 (stores still in L2 at kernel end) (profiles/decode_split_kernel_config3.md)"}
TRAFFIC_SCALEOUT = {"bytes_per_launch_per_bank": 14_435,
                    "source": "ncu at 224 requests (12,544 banks, prefix 256): cow_count_kernel 8.57 MB + "
                              "cow_decode_kernel 172.5 MB per step, scaled by banks "
                              "(profiles/decode_kernel_config4_hashed.md)"}


def algorithmic_bytes(banks: int, first_touches: int, *, idx_bytes=8, val_bytes=4, act_bytes=4) -> int:
    """Per-launch algorithmic bytes of the fused step (all pools).

    Per (bank, layer, token): D*s_v*(2W+R) row traffic + D*(s_in+s_out)
    value/readout + (W+R)*(s_idx + 4 + s_w) routes/map/weights + 3*s_g + 8
    gates and template; plus 8 bytes per first touch (stack read + map store).
    """
    per = (WIDTH * val_bytes * (2 * WRITES + READS) + WIDTH * 2 * act_bytes
           + (WRITES + READS) * (idx_bytes + 4 + act_bytes) + 3 * act_bytes + 8)
    return banks * per + 8 * first_touches


def dense_algorithmic_bytes(banks: int) -> int:
    per = (WIDTH * 4 * (2 * WRITES + READS) + WIDTH * 2 * 4 + (WRITES + READS) * (8 + 4) + 3 * 4)
    return banks * per


# --------------------------------------------------------------------------
# synthetic inputs
# --------------------------------------------------------------------------


def uniform_routes(gen: torch.Generator, shape, k: int, device) -> torch.Tensor:
    keys = torch.rand(*shape, SLOTS, generator=gen, device=device)
    return keys.argsort(dim=-1)[..., :k].contiguous()


def step_inputs(gen, banks, steps, device):
    """Decode inputs for ``steps`` tokens and all layers: dict of [S, L, banks, ...]."""
    shape = (steps, LAYERS, banks)
    return dict(
        write_indices=uniform_routes(gen, shape, WRITES, device),
        write_weights=torch.softmax(torch.randn(*shape, WRITES, generator=gen, device=device), -1),
        values=torch.randn(*shape, WIDTH, generator=gen, device=device),
        input_gate=torch.rand(*shape, generator=gen, device=device),
        forget_log_gate=-torch.rand(*shape, generator=gen, device=device),
        read_indices=uniform_routes(gen, shape, READS, device),
        read_weights=torch.softmax(torch.randn(*shape, READS, generator=gen, device=device), -1),
    )


def prefill_pools(gen, banks, device, prefix=PREFIX):
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState

    q = max(16, banks * WRITES * QUANTUM_STEPS)
    states = []
    for _ in range(LAYERS):
        m0 = 0.02 * torch.randn(HEADS, SLOTS, WIDTH, generator=gen, device=device)
        shape = (banks, prefix)
        st, _ = PackedSDMCopyOnWriteState.from_prefix_routes(
            m0,
            uniform_routes(gen, shape, WRITES, device),
            torch.softmax(torch.randn(*shape, WRITES, generator=gen, device=device), -1),
            torch.randn(*shape, WIDTH, generator=gen, device=device),
            torch.rand(*shape, generator=gen, device=device),
            -torch.rand(*shape, generator=gen, device=device),
            uniform_routes(gen, shape, READS, device),
            torch.softmax(torch.randn(*shape, READS, generator=gen, device=device), -1),
            template_indices=torch.zeros(banks, dtype=torch.int64, device=device),
            growth_quantum_rows=q,
        )
        states.append(st)
    return states


# --------------------------------------------------------------------------
# clocks
# --------------------------------------------------------------------------


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------


def _c_step(inputs, s, l, outputs):
    from copy_on_write_sdm_b200 import _lib

    def p(name):
        return inputs[name][s, l].data_ptr()

    return _lib.CowStep(p("write_indices"), p("write_weights"), p("values"), p("input_gate"),
                        p("input_gate"), p("forget_log_gate"), p("read_indices"), p("read_weights"),
                        outputs[l].data_ptr(), None)


def _sum_state_bytes(states) -> dict:
    out = {}
    for st in states:
        for k, v in st.storage_bytes().items():
            out[k] = out.get(k, 0) + v
    return out


def run_gpu(args, rank, world, device, *, batch=BATCH, prefix=PREFIX, extras=True):
    """Configuration 3 on this rank: ``batch`` requests, ``prefix`` prefill tokens.

    ``extras`` adds the warm-L2 trace, the single-launch timing and the
    end-to-end legs; without it the flushed device trace, the dense control
    and the incremental graph timing run (the sub-legs of the default run)."""
    from copy_on_write_sdm_b200 import _lib, allocator, packed_sdm_cow_step_layers, dense_sdm_sparse_step_layers

    lib = _lib.load()
    gen = torch.Generator(device=device).manual_seed(1000 + rank + 17 * prefix)
    banks = batch * HEADS
    K, Wm = args.steps, args.warmup
    t_setup = time.time()
    states = prefill_pools(gen, banks, device, prefix)
    inputs = step_inputs(gen, banks, K + Wm, device)
    torch.cuda.synchronize(device)
    setup_s = time.time() - t_setup

    # Warm-up steps through the public API (capacity proof + growth as in serving).
    for s in range(Wm):
        for st in states:
            st.prepare_step_capacity(banks * WRITES)
        packed_sdm_cow_step_layers(states, [{k: v[s, l] for k, v in inputs.items()} for l in range(LAYERS)])
    # Prove capacity for every timed step up front (pessimistic: W first touches per bank-step).
    for st in states:
        st.prepare_step_capacity(banks * WRITES * K)
    free_before = sum(int(st.free_count) for st in states)
    for st in states:
        st.validate_invariants()

    outputs = [torch.empty(banks, WIDTH, device=device) for _ in range(LAYERS)]
    scratch = allocator.decode_scratch(device, banks * LAYERS, LAYERS)
    pools = (_lib.CowPool * LAYERS)(*[st._pool() for st in states])
    stream = torch.cuda.Stream(device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    step_structs = {s: (_lib.CowStep * LAYERS)(*[_c_step(inputs, s, l, outputs) for l in range(LAYERS)])
                    for s in range(Wm, Wm + K)}

    def packed_launch(s):
        _lib.check(lib.cow_decode_step(pools, step_structs[s], LAYERS, WRITES, READS, _lib.I64, _lib.F32,
                                       scratch.data_ptr(), scratch.numel(), stream.cuda_stream), "cow_decode_step")

    def flushed_trace(launch):
        """ONE graph of K x (L2 flush, event, step, event): every step starts with a
        cold L2 and is timed on the device by its own event pair, with no host
        submission gap inside any interval."""
        evs = [(torch.cuda.Event(enable_timing=True, external=True),
                torch.cuda.Event(enable_timing=True, external=True)) for _ in range(K)]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for i, s in enumerate(range(Wm, Wm + K)):
                    flush.fill_(float(i))
                    evs[i][0].record(stream)
                    launch(s)
                    evs[i][1].record(stream)
        return g, evs

    # The timed trace: K steps in ONE graph between one event pair, step i on
    # replica i mod REPLICAS of the pools (independent copies of this rank's
    # state, taken after the warm-up).  Between two visits of a replica the
    # other replicas' steps move ~5.5 MB each, more than twice the 126 MB L2,
    # so every step starts cold without a flush, and no event node sits
    # between two steps (an event pair around each microsecond-scale step adds
    # its own ~4.5 us of graph scheduling to the interval: the flushed
    # per-step figure below keeps that timing for comparison).
    replicas = []
    for _ in range(REPLICAS):
        arr, keep = (_lib.CowPool * LAYERS)(), []
        for l, st in enumerate(states):
            pool = st._pool()
            t = dict(m0=st._m0_f32.clone(), templates=st.template_indices.clone(), slab=st.values.clone(),
                     map=st.logical_to_physical.clone(), free_rows=st.free_rows.clone(),
                     free_count=st.free_count.clone(), status=st.overflow_flag.clone())
            for name, v in t.items():
                setattr(pool, name, v.data_ptr())
            arr[l] = pool
            keep.append(t)
        replicas.append((arr, keep))

    def replica_free() -> int:
        return sum(int(t["free_count"]) for _, keep in replicas for t in keep)

    rgraph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(rgraph, stream=stream):
            for i, s in enumerate(range(Wm, Wm + K)):
                _lib.check(lib.cow_decode_step(replicas[i % REPLICAS][0], step_structs[s], LAYERS, WRITES, READS,
                                               _lib.I64, _lib.F32, scratch.data_ptr(), scratch.numel(),
                                               stream.cuda_stream), "cow_decode_step")
    # Upload the graph before the timed replay (a warm-up replay would make
    # the timed one re-apply the same routes, so no step would allocate).
    ctypes.CDLL("libcuda.so.1").cuGraphUpload(ctypes.c_void_p(rgraph.raw_cuda_graph_exec()),
                                              ctypes.c_void_p(stream.cuda_stream))
    torch.cuda.synchronize(device)
    rfree_before = replica_free()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graph, ev = flushed_trace(packed_launch)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    with ClockSampler(device.index) as clocks:
        barrier()
        torch.cuda.synchronize(device)
        with torch.cuda.stream(stream):
            r0.record(stream)
            rgraph.replay()
            r1.record(stream)
        torch.cuda.synchronize(device)
        barrier()
    total_ms = r0.elapsed_time(r1)
    first_touches = rfree_before - replica_free()
    # The flushed per-step trace on the pools themselves (one event pair per step).
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize(device)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    flushed_ms = sum(step_ms)
    flushed_first_touches = free_before - sum(int(st.free_count) for st in states)
    for st in states:
        st.validate_invariants()
    del replicas

    # Each step as its own graph launch, timed alone (adds the host submission
    # latency of every launch to its interval): the single-token latency.
    single = []
    with torch.cuda.stream(stream):
        for s in (range(Wm, Wm + min(K, 16)) if extras else ()):
            g1 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1, stream=stream):
                packed_launch(s)
            flush.fill_(float(s))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g1.replay()
            e1.record(stream)
            torch.cuda.synchronize(device)
            single.append(e0.elapsed_time(e1))
    single_ms = statistics.median(single) if single else None

    # Warm-L2 trace: all K steps captured in ONE graph and replayed back to
    # back (no host in the loop; the pool state stays L2-resident).  The
    # routes are re-applied to the evolved state; with every slot of every
    # bank already private nothing is allocated.
    warm = dense_warm = dense_ms = incremental = eager = None
    if rank == 0:
        def trace_graph(launch):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    for s in range(Wm, Wm + K):
                        launch(s)
            return g

        def time_graph(g):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                g.replay()  # warm the graph itself
                torch.cuda.synchronize(device)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize(device)
            return e0.elapsed_time(e1)

        warm = time_graph(trace_graph(packed_launch)) if extras else None

        # Dense-table control, same routes, same timing disciplines.
        mems = [st.materialize_dense() for st in states]
        dptrs = (ctypes.c_void_p * LAYERS)(*[m.data_ptr() for m in mems])
        dbanks = (ctypes.c_int64 * LAYERS)(*([banks] * LAYERS))

        def dense_launch(s):
            _lib.check(lib.cow_dense_step(dptrs, dbanks, step_structs[s], LAYERS, SLOTS, WIDTH, _lib.F32, WRITES,
                                          READS, _lib.I64, _lib.F32, stream.cuda_stream), "cow_dense_step")

        dense_warm = time_graph(trace_graph(dense_launch)) if extras else None
        dgraph, dev_ev = flushed_trace(dense_launch)
        with torch.cuda.stream(stream):
            dgraph.replay()
        torch.cuda.synchronize(device)
        dense_ms = sum(a.elapsed_time(b) for a, b in dev_ev)

        # Incremental device time of a cold step inside a graph: a graph of
        # K x (flush, step) against a graph of K x flush.  Event nodes around a
        # microsecond-scale kernel add their own scheduling to its interval;
        # the difference of two whole-graph times does not.
        def flushed_only(launch):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    for i, s in enumerate(range(Wm, Wm + K)):
                        flush.fill_(float(i))
                        if launch is not None:
                            launch(s)
            return g

        # The same flushed steps launched eagerly, each between its own event
        # pair on the launching stream (the 256 MiB flush before each step
        # keeps the host's submissions ahead of the device, so no host gap
        # falls inside an interval).
        def eager_flushed(launch):
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
            with torch.cuda.stream(stream):
                for i, s in enumerate(range(Wm, Wm + K)):
                    flush.fill_(float(i))
                    evs[i][0].record(stream)
                    launch(s)
                    evs[i][1].record(stream)
            torch.cuda.synchronize(device)
            return 1e3 * sum(a.elapsed_time(b) for a, b in evs) / K

        eager = None
        if extras:
            eager = {"packed_us": eager_flushed(packed_launch), "dense_us": eager_flushed(dense_launch)}
        base = time_graph(flushed_only(None))
        # The incremental graphs re-apply the K steps twice more to the evolved
        # pools: prove capacity for them (pools whose slots are all private pop nothing).
        for st in states:
            st.prepare_step_capacity(banks * WRITES * 2 * K)
        # A proof may have grown a slab into a new store: the launches below
        # must see the pools' current tensors.
        pools = (_lib.CowPool * LAYERS)(*[st._pool() for st in states])
        tiny = torch.zeros(1, device=device)
        incremental = {"empty_kernel_us": 1e3 * (time_graph(flushed_only(lambda s: tiny.add_(1.0))) - base) / K,
                       "packed_us": 1e3 * (time_graph(flushed_only(packed_launch)) - base) / K,
                       "dense_us": 1e3 * (time_graph(flushed_only(dense_launch)) - base) / K}
        del mems

    if not extras:
        return dict(total_ms=total_ms, step_ms=step_ms, flushed_ms=flushed_ms, flushed_first_touches=flushed_first_touches,
                    dense_ms=dense_ms, incremental=incremental,
                    first_touches=first_touches, clocks=clocks.summary(), setup_s=setup_s, banks=banks,
                    state_bytes=_sum_state_bytes(states))

    # End to end through the public runtime API with host buffers: every step
    # copies its packed routes from pinned host memory (one copy), runs the
    # capacity proof and the fused launch (DecodeSession), and reads the
    # readouts back to pinned host memory (one copy).
    from copy_on_write_sdm_b200 import DecodeSession

    # Capacity is proven for every end-to-end step up front, as for the timed
    # device trace (growing the slab by whole quanta now): each step still runs
    # the per-step proof (one decrement per pool), but no step has to
    # reconcile with the device's free count in the middle of the stream.
    for st in states:
        st.prepare_step_capacity(banks * WRITES * (4 * K + 4 * E2E_WARMUP))
    sess = DecodeSession(states, writes=WRITES, reads=READS)
    host_steps = torch.empty(K, sess.step_bytes, dtype=torch.uint8, pin_memory=True)
    for i, s in enumerate(range(Wm, Wm + K)):
        for l in range(LAYERS):
            for k, v in sess.views[l].items():
                v.copy_(inputs[k][s, l])
        host_steps[i].copy_(sess.inputs)
    torch.cuda.synchronize(device)
    sess.register_host_steps(host_steps)
    h2d = sess.step_bytes
    d2h = sess.host_outputs.numel() * sess.host_outputs.element_size()
    # The host-to-host legs run on the device's default stream, the stream a
    # serving process that never creates one submits to (its runtime calls
    # cost the host measurably less there than on a created stream).
    host_stream = torch.cuda.default_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(device)
    with torch.cuda.stream(host_stream):
        e0.record(host_stream)
        for i in range(K):
            sess.step_host(host_steps[i])
        e1.record(host_stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_serial_ms = e0.elapsed_time(e1)
    # The same through step_host_pipelined: step k+1's input copy and step
    # k-1's readout copy overlap step k's decode (three streams, in-order decode).
    with torch.cuda.stream(host_stream):
        for i in range(E2E_WARMUP):  # warm-up: side streams, buffers, a steady host/device rhythm
            sess.step_host_pipelined(host_steps[i % K])
    torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)
    with torch.cuda.stream(host_stream):
        e0.record(host_stream)
        last = None
        t0 = time.perf_counter()
        for i in range(K):
            _, last = sess.step_host_pipelined(host_steps[i])
        piped_host_s = time.perf_counter() - t0
        host_stream.wait_event(last)
        e1.record(host_stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    # The same through step_host_mapped: the decode kernel reads each step's
    # pinned host bytes and writes its readouts to pinned host memory itself
    # (zero-copy over PCIe): one launch per token, no copy calls.
    with torch.cuda.stream(host_stream):
        for i in range(E2E_WARMUP):
            sess.step_host_mapped(host_steps[i % K])
    torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)
    with torch.cuda.stream(host_stream):
        e0.record(host_stream)
        t0 = time.perf_counter()
        for i in range(K):
            sess.step_host_mapped(host_steps[i])
        host_s = time.perf_counter() - t0
        e1.record(host_stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_mapped_ms = e0.elapsed_time(e1)
    # Device time of the same zero-copy launches with no host in the loop (one
    # CUDA graph of K mapped steps): separates PCIe / kernel time from host time.
    for st in states:  # prove the two replays below up front (the graph bakes the pool tensors in)
        st.prepare_step_capacity(banks * WRITES * 2 * K)
    with torch.cuda.stream(stream):
        sess.step_host_mapped(host_steps[0])  # refreshes the descriptors' pool array
    torch.cuda.synchronize(device)
    pipe = sess._pipeline()
    gdescs = []
    for d in pipe["descs"]:  # the same descriptors without the arrival event (nothing to record in a graph)
        g = _lib.CowHostPipeline()
        ctypes.memmove(ctypes.addressof(g), ctypes.addressof(d), ctypes.sizeof(g))
        g.d2h_done = None
        gdescs.append(g)
    mapped_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(mapped_graph, stream=stream):
            for i in range(K):
                b = i & 1
                _lib.check(lib.cow_decode_step_host_mapped(ctypes.addressof(gdescs[b]), host_steps[i].data_ptr(),
                                                           pipe["host_outputs"][b].data_ptr(), stream.cuda_stream),
                           "cow_decode_step_host_mapped")
        mapped_graph.replay()
        torch.cuda.synchronize(device)
        e0.record(stream)
        mapped_graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(device)
    mapped_device = {"us_per_step": 1e3 * e0.elapsed_time(e1) / K, "host_us_per_step": 1e6 * host_s / K,
                     "note": "us_per_step: K mapped launches replayed as one CUDA graph (no host in the loop); "
                             "host_us_per_step: host time of the step_host_mapped calls in the e2e loop"}

    state_bytes = _sum_state_bytes(states)
    used = [st.used_bytes() for st in states]
    return dict(total_ms=total_ms, step_ms=step_ms, flushed_ms=flushed_ms, flushed_first_touches=flushed_first_touches,
                single_ms=single_ms, e2e_ms=e2e_ms, e2e_serial_ms=e2e_serial_ms,
                piped_host_us=1e6 * piped_host_s / K,
                e2e_mapped_ms=e2e_mapped_ms, mapped_device=mapped_device, eager=eager,
                warm_ms=warm, incremental=incremental,
                dense_ms=dense_ms,
                dense_warm_ms=dense_warm,
                first_touches=first_touches, h2d=h2d, d2h=d2h, clocks=clocks.summary(), setup_s=setup_s,
                state_bytes=state_bytes, live_value_bytes=sum(u["live_value_bytes"] for u in used),
                allocated_rows=sum(u["allocated_rows"] for u in used),
                capacity_rows=sum(st.capacity_rows for st in states))


# --------------------------------------------------------------------------
# configuration 4: large-address-space scale-out (--workload scaleout)
# --------------------------------------------------------------------------

SO_SLOTS, SO_HEADS, SO_REQUESTS, SO_PREFIX, SO_ZIPF = 65536, 8, 1024, 4096, 1.1


class ZipfRoutes:
    """Zipf(s) popularity over a seeded permutation of the N addresses."""

    def __init__(self, n: int, s: float, gen: torch.Generator, device):
        ranks = torch.arange(1, n + 1, device=device, dtype=torch.float64)
        p = ranks.pow(-s)
        p /= p.sum()
        self.n = n
        self.cdf = torch.cumsum(p, 0).float()
        self.logp = p.log().float()
        self.perm = torch.randperm(n, generator=gen, device=device)

    def with_replacement(self, shape, gen) -> torch.Tensor:
        u = torch.rand(*shape, generator=gen, device=self.cdf.device)
        return self.perm[torch.searchsorted(self.cdf, u).clamp_(max=self.n - 1)]

    def distinct(self, rows: int, k: int, gen, chunk: int = 2048) -> torch.Tensor:
        """``k`` distinct addresses per row, without replacement (Gumbel top-k)."""
        out = []
        for r0 in range(0, rows, chunk):
            r = min(chunk, rows - r0)
            g = torch.rand(r, self.n, generator=gen, device=self.cdf.device).clamp_(min=1e-20)
            g.log_().neg_().log_().neg_().add_(self.logp)
            out.append(self.perm[g.topk(k, dim=-1).indices])
            del g
        return torch.cat(out)


def scaleout_pool(gen, requests: int, prefix: int, extra_rows: int, device):
    """Post-prefix pool of one configuration-4 layer.

    The written-address union of ``prefix`` Zipf-routed tokens (W=4 writes each)
    is marked and packed in ``nonzero()`` order exactly as the prefill handoff
    does; the touched rows hold M0 instead of the recurrence's values (the
    4,096-token recurrence over 8,192 banks would dominate the run and its
    inputs alone are ~17 GB per layer).  Decode traffic does not depend on row
    contents.  Capacity: the touched rows + ``extra_rows`` (proven, no growth).
    """
    from copy_on_write_sdm_b200 import PackedSDMCopyOnWriteState, _lib

    lib = _lib.load()
    banks = requests * SO_HEADS
    zipf = ZipfRoutes(SO_SLOTS, SO_ZIPF, gen, device)
    m0 = 0.02 * torch.randn(SO_HEADS, SO_SLOTS, WIDTH, generator=gen, device=device)
    mapping = torch.full((banks, SO_SLOTS), -1, dtype=torch.int32, device=device)
    status = torch.zeros((), dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    chunk = 256
    for t0 in range(0, prefix, chunk):
        t = min(chunk, prefix - t0)
        widx = zipf.with_replacement((banks, t, WRITES), gen)
        _lib.check(lib.cow_prefill_mark(widx.data_ptr(), _lib.I64, banks, t, WRITES, SO_SLOTS, mapping.data_ptr(),
                                        status.data_ptr(), stream), "cow_prefill_mark")
        del widx
    touched = int((mapping >= 0).sum())
    templates = torch.arange(SO_HEADS, device=device, dtype=torch.int64).repeat(requests)
    st = PackedSDMCopyOnWriteState._pack_layout(
        m0, mapping, templates, capacity_rows=touched + extra_rows, state_dtype=torch.float32,
        maximum_future_allocations=extra_rows, growth_quantum_rows=0, row_source=("m0", None), validate=False)
    return st, zipf, touched


def run_gpu_scaleout(args, rank, world, device):
    from copy_on_write_sdm_b200 import _lib, allocator

    lib = _lib.load()
    requests = args.requests // world
    banks = requests * SO_HEADS
    K, Wm = args.steps, args.warmup
    gen = torch.Generator(device=device).manual_seed(4000 + rank)
    t0 = time.time()
    hashed_leg = getattr(args, "hash_leg", False)
    total_steps = K + Wm + (K if hashed_leg else 0)
    states, zipfs, touched = [], [], []
    for _ in range(LAYERS):
        st, z, a = scaleout_pool(gen, requests, args.prefix, banks * WRITES * total_steps, device)
        states.append(st)
        zipfs.append(z)
        touched.append(a)
    steps = []
    for s in range(total_steps):
        per = []
        for l in range(LAYERS):
            z = zipfs[l]
            per.append(dict(
                write_indices=z.distinct(banks, WRITES, gen), read_indices=z.distinct(banks, READS, gen),
                write_weights=torch.softmax(torch.randn(banks, WRITES, generator=gen, device=device), -1),
                read_weights=torch.softmax(torch.randn(banks, READS, generator=gen, device=device), -1),
                values=torch.randn(banks, WIDTH, generator=gen, device=device),
                input_gate=torch.rand(banks, generator=gen, device=device),
                forget_log_gate=-torch.rand(banks, generator=gen, device=device)))
        steps.append(per)
    torch.cuda.synchronize(device)
    setup_s = time.time() - t0
    outputs = [torch.empty(banks, WIDTH, device=device) for _ in range(LAYERS)]
    scratch = allocator.decode_scratch(device, banks * LAYERS, LAYERS)
    pools = (_lib.CowPool * LAYERS)(*[st._pool() for st in states])

    def cstep(x, out):
        return _lib.CowStep(x["write_indices"].data_ptr(), x["write_weights"].data_ptr(), x["values"].data_ptr(),
                            x["input_gate"].data_ptr(), x["input_gate"].data_ptr(), x["forget_log_gate"].data_ptr(),
                            x["read_indices"].data_ptr(), x["read_weights"].data_ptr(), out.data_ptr(), None)

    c_steps = [(_lib.CowStep * LAYERS)(*[cstep(steps[s][l], outputs[l]) for l in range(LAYERS)])
               for s in range(total_steps)]
    stream = torch.cuda.Stream(device)

    def launch(s):
        _lib.check(lib.cow_decode_step(pools, c_steps[s], LAYERS, WRITES, READS, _lib.I64, _lib.F32,
                                       scratch.data_ptr(), scratch.numel(), stream.cuda_stream), "cow_decode_step")

    with torch.cuda.stream(stream):
        for s in range(Wm):
            launch(s)
    torch.cuda.synchronize(device)
    free_before = sum(int(st.free_count) for st in states)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    with ClockSampler(device.index) as clocks:
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        with torch.cuda.stream(stream):
            for i in range(K):
                ev[i][0].record(stream)
                launch(Wm + i)
                ev[i][1].record(stream)
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    first = free_before - sum(int(st.free_count) for st in states)
    state_bytes = _sum_state_bytes(states)
    hashed = None
    if hashed_leg:
        # The same pools on hashed maps (tables sized for every bank's private
        # slots plus the remaining steps' first touches), timed on the next K
        # steps of the trace.
        if getattr(args, "hash_max_load", 0.0):
            type(states[0]).HASH_MAX_LOAD = args.hash_max_load
        for st in states:
            st.use_hash_map(headroom_rows_per_bank=WRITES * K)
        torch.cuda.empty_cache()
        pools = (_lib.CowPool * LAYERS)(*[st._pool() for st in states])
        free_h = sum(int(st.free_count) for st in states)
        evh = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
        torch.cuda.synchronize(device)
        with torch.cuda.stream(stream):
            for i in range(K):
                evh[i][0].record(stream)
                launch(Wm + K + i)
                evh[i][1].record(stream)
        torch.cuda.synchronize(device)
        hms = [a.elapsed_time(b) for a, b in evh]
        hashed = {"total_ms": sum(hms), "first_touches": free_h - sum(int(st.free_count) for st in states),
                  "table_slots": [st.map_table_slots for st in states],
                  "map_bytes": sum(st.storage_bytes()["logical_to_physical"] for st in states),
                  "dense_map_bytes": state_bytes["logical_to_physical"],
                  "status": sum(st.status() for st in states)}
    for st in states:
        st.validate_invariants()
    return dict(total_ms=sum(step_ms), step_ms=step_ms, first_touches=first, clocks=clocks.summary(),
                setup_s=setup_s, state_bytes=state_bytes, requests=requests, banks=banks, hashed=hashed,
                mean_touched_rows_per_bank=sum(touched) / (LAYERS * banks))


def cpu_scaleout_rate(seconds: float, requests: int, prefix: int) -> dict:
    """Oracle packed step on 8 requests (64 banks) of one configuration-4 layer,
    extrapolated to ``requests`` x 7 layers per decode step (bank-steps are
    independent, so CPU time scales with their number)."""
    from oracle import cow_oracle as O

    rng = np.random.default_rng(11)
    sample_req = 8
    banks = sample_req * SO_HEADS
    ranks = np.arange(1, SO_SLOTS + 1, dtype=np.float64)
    p = ranks ** -SO_ZIPF
    p /= p.sum()
    cdf = np.cumsum(p)
    perm = rng.permutation(SO_SLOTS)
    touched = np.zeros((banks, SO_SLOTS), bool)
    for b in range(banks):
        touched[b, perm[np.minimum(np.searchsorted(cdf, rng.random(prefix * WRITES)), SO_SLOTS - 1)]] = True
    m0 = (0.02 * rng.standard_normal((SO_HEADS, SO_SLOTS, WIDTH))).astype(np.float32)
    st = O.allocate(m0, banks=banks, capacity_rows=int(touched.sum()) + banks * WRITES * 64,
                    template_indices=np.tile(np.arange(SO_HEADS), sample_req))
    bank, slot = np.nonzero(touched)
    st.logical_to_physical[bank, slot] = np.arange(bank.size, dtype=np.int32)
    cap = st.capacity_rows
    st.free_rows[: cap - bank.size] = np.arange(bank.size, cap, dtype=np.int32)
    st.free_count = cap - bank.size

    def draw(k):
        keys = np.log(p)[None, :] - np.log(-np.log(rng.random((banks, SO_SLOTS))))
        return perm[np.argpartition(-keys, k, axis=1)[:, :k]]

    xs = []
    for _ in range(4):
        x = O.synthetic_step_inputs(rng, banks, 16, WIDTH, WRITES, READS)
        x["write_indices"], x["read_indices"] = draw(WRITES), draw(READS)
        xs.append(x)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        O.packed_step(st, **xs[n % len(xs)])
        n += 1
    per_bank_step = (time.perf_counter() - t0) / (n * banks)
    step_s = per_bank_step * requests * SO_HEADS * LAYERS
    return {"value": requests / step_s, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n} oracle steps of {banks} banks (8 requests x 8 heads, N=65536, Zipf 1.1, prefix {prefix}) "
                      f"on one layer, extrapolated to {requests} requests x {LAYERS} layers per decode step"}


# --------------------------------------------------------------------------
# Configuration 5: continuous-batching churn
# --------------------------------------------------------------------------

CH_SLOTS, CH_HEADS, CH_LIVE, CH_ARRIVALS = 4096, 4, 256, 8.0
CH_MIN_LEN, CH_MAX_LEN, CH_PROMPT, CH_WARM_PREFIX = 64, 4096, 64, 1024


def affine_routes(gen, lead: tuple, k: int, n: int, device) -> torch.Tensor:
    """``k`` distinct uniform addresses per row: ``(base + stride*j) mod n`` with a
    uniform base and a uniform odd stride (``n`` is a power of two, so the k
    addresses are distinct and each is marginally uniform over ``[0, n)``)."""
    base = torch.randint(0, n, lead + (1,), generator=gen, device=device)
    stride = 2 * torch.randint(0, n // 2, lead + (1,), generator=gen, device=device) + 1
    return (base + stride * torch.arange(k, device=device)) % n


def churn_prompts(gen, requests: int, tokens: int, device) -> list[dict]:
    """Seeded prompt routes, values and gates of ``requests`` requests, one dict per layer."""
    banks = requests * CH_HEADS
    return [dict(
        write_indices=affine_routes(gen, (banks, tokens), WRITES, CH_SLOTS, device),
        write_weights=torch.softmax(torch.randn(banks, tokens, WRITES, generator=gen, device=device), -1),
        values=torch.randn(banks, tokens, WIDTH, generator=gen, device=device),
        input_gate=torch.rand(banks, tokens, generator=gen, device=device),
        forget_log_gate=-torch.rand(banks, tokens, generator=gen, device=device),
        read_indices=affine_routes(gen, (banks, tokens), READS, CH_SLOTS, device),
        read_weights=torch.softmax(torch.randn(banks, tokens, READS, generator=gen, device=device), -1))
        for _ in range(LAYERS)]


def churn_prefill(m0s, prompts: list[dict], first: int, requests: int, quantum: int):
    """Prefilled cohort of requests ``first .. first+requests-1`` of ``prompts`` (all
    layers in one sparse-prefill call), as ``FaithfulSDMDecodeState``."""
    from copy_on_write_sdm_b200.allocator import from_prefix_routes_layers
    from copy_on_write_sdm_b200.inference import FaithfulSDMDecodeState

    lo, hi = first * CH_HEADS, (first + requests) * CH_HEADS
    device = m0s[0].device
    templates = torch.arange(CH_HEADS, device=device, dtype=torch.int64).repeat(requests)
    states, _ = from_prefix_routes_layers(m0s, [{k: v[lo:hi] for k, v in x.items()} for x in prompts],
                                          template_indices=templates, growth_quantum_rows=quantum)
    tokens = prompts[0]["values"].shape[1]
    return FaithfulSDMDecodeState(
        layout="B" * LAYERS, position=tokens, capacity=0, activation_dtype=torch.float32,
        active_sequences=torch.ones(requests, dtype=torch.bool, device=device),
        sdm_layer_positions=tuple(range(LAYERS)), sdm_states=tuple(states), dense_keys=(), dense_values=())


def churn_admit_prefix(state, prompts: list[dict], first: int, requests: int) -> None:
    """Requests ``first .. first+requests-1`` of ``prompts`` prefilled straight into
    the live pools of ``state`` (``FaithfulSDMDecodeState.admit_prefix``)."""
    lo, hi = first * CH_HEADS, (first + requests) * CH_HEADS
    device = state.device
    templates = torch.arange(CH_HEADS, device=device, dtype=torch.int64).repeat(requests)
    state.admit_prefix([{k: v[lo:hi] for k, v in x.items()} for x in prompts], template_indices=templates)


def run_gpu_churn(args, rank, world, device):
    """Continuous batching over 256 live slots per GPU.

    Every step: requests whose decode length ran out are released and the
    batch compacted (``release_and_compact``), a cohort of the same size is
    prefilled (64-token prompts, sparse prefill) and admitted (``admit``),
    the slab is trimmed every ``--trim-every`` steps if asked, each pool's
    then ``DecodeSession.step`` renews each pool's capacity proof
    (``prepare_step_capacity``, growing by whole quanta) and runs one fused
    decode launch over the 7 pools.  Arrivals are
    Poisson(8) per step into a FIFO queue; with mean length 2,080 tokens the
    queue never drains, so the batch stays full and admissions equal
    completions.  The initial batch starts from a 1,024-token prefix (about
    2,600 private rows per bank, near the steady-state mean) with residual
    lengths drawn uniformly below each request's length.
    """
    from copy_on_write_sdm_b200 import DecodeSession

    rng = np.random.default_rng(5000 + rank)
    gen = torch.Generator(device=device).manual_seed(5000 + rank)
    live = CH_LIVE
    banks = live * CH_HEADS
    quantum = max(16, banks * WRITES * args.quantum_steps)
    K, Wm = args.steps, args.warmup
    t0 = time.time()
    m0s = [0.02 * torch.randn(CH_HEADS, CH_SLOTS, WIDTH, generator=gen, device=device) for _ in range(LAYERS)]
    state = churn_prefill(m0s, churn_prompts(gen, live, args.churn_warm_prefix, device), 0, live, quantum)
    ring_requests = 64
    prompts = churn_prompts(gen, ring_requests, CH_PROMPT, device)
    next_prompt = 0
    lengths = rng.integers(CH_MIN_LEN, CH_MAX_LEN + 1, size=live)
    remaining = np.array([rng.integers(1, n + 1) for n in lengths])
    # Decode runs through a DecodeSession over the state's pools (the objects
    # persist through release/compact/admit/trim; the session re-reads their
    # tensors when they change).  Each step's routes are one device copy from
    # a ring of 16 pre-generated steps into the session's input buffer.
    session = DecodeSession(state.sdm_states, writes=WRITES, reads=READS)
    ring = []
    for _ in range(16):
        for v in session.views:
            v["write_indices"].copy_(affine_routes(gen, (banks,), WRITES, CH_SLOTS, device))
            v["read_indices"].copy_(affine_routes(gen, (banks,), READS, CH_SLOTS, device))
            v["write_weights"].copy_(torch.softmax(torch.randn(banks, WRITES, generator=gen, device=device), -1))
            v["read_weights"].copy_(torch.softmax(torch.randn(banks, READS, generator=gen, device=device), -1))
            v["values"].copy_(torch.randn(banks, WIDTH, generator=gen, device=device))
            v["input_gate"].copy_(torch.rand(banks, generator=gen, device=device))
            v["forget_log_gate"].copy_(-torch.rand(banks, generator=gen, device=device))
        ring.append(session.inputs.clone())
    # Untimed completion cycles (release, compact, cohort prefill, admit):
    # the first call of each lifecycle kernel pays the module load and its
    # workspace allocations (tens of milliseconds), which is start-up, not churn.
    for n in (1, 2):  # two sizes: some kernels first run at the second
        state.release_and_compact(list(range(n)))
        if args.churn_admit == "prefix":
            churn_admit_prefix(state, prompts, 0, n)
        else:
            state.admit(churn_prefill(m0s, prompts, 0, n, quantum))
        remaining = np.concatenate([remaining[n:], rng.integers(CH_MIN_LEN, CH_MAX_LEN + 1, size=n)])
    torch.cuda.synchronize(device)
    setup_s = time.time() - t0
    stats = dict(completions=0, released_rows=0, trimmed_rows=0, queue=0)
    admitted_rows = []  # device counts, read after the timed region
    stream = torch.cuda.current_stream(device)

    def one_step(s, timed, ev):
        nonlocal remaining, next_prompt
        if timed:
            ev[0].record(stream)
        stats["queue"] += int(rng.poisson(CH_ARRIVALS))
        done = np.nonzero(remaining == 0)[0]
        if done.size:
            stats["completions"] += done.size
            stats["queue"] -= done.size
            stats["released_rows"] += state.release_and_compact(done.tolist())
            if next_prompt + done.size > ring_requests:
                next_prompt = 0
            if args.churn_admit == "prefix":
                # prefill straight into the live pools (admit_prefix)
                before = torch.stack([st.allocated_rows_tensor() for st in state.sdm_states]).sum()
                churn_admit_prefix(state, prompts, next_prompt, int(done.size))
                admitted_rows.append(torch.stack([st.allocated_rows_tensor() for st in state.sdm_states]).sum()
                                     - before)
            else:
                cohort = churn_prefill(m0s, prompts, next_prompt, int(done.size), quantum)
                admitted_rows.append(torch.stack([st.allocated_rows_tensor() for st in cohort.sdm_states]).sum())
                state.admit(cohort)
            next_prompt += int(done.size)
            remaining = np.concatenate([remaining[remaining > 0],
                                        rng.integers(CH_MIN_LEN, CH_MAX_LEN + 1, size=done.size)])
        if args.trim_every and s % args.trim_every == args.trim_every - 1:
            stats["trimmed_rows"] += state.trim_sdm_pools(headroom_rows=banks * WRITES)
        if timed:
            ev[1].record(stream)
        session.inputs.copy_(ring[s % len(ring)])
        session.step()
        if timed:
            ev[2].record(stream)
        remaining = remaining - 1

    for s in range(Wm):
        one_step(s, False, None)
    torch.cuda.synchronize(device)
    growth0 = [(st.growth_events, st.growth_rows_added, st.growth_rows_copied) for st in state.sdm_states]
    for k in stats:
        stats[k] = 0
    admitted_rows.clear()
    ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(K)]
    with ClockSampler(device.index) as clocks:
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        for i in range(K):
            one_step(Wm + i, True, ev[i])
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
    stats["admitted_rows"] = int(sum(int(x) for x in admitted_rows))
    life_ms = [a.elapsed_time(b) for a, b, _ in ev]
    dec_ms = [b.elapsed_time(c) for _, b, c in ev]
    for st in state.sdm_states:
        st.validate_invariants()
    growth = [tuple(x - y for x, y in zip((st.growth_events, st.growth_rows_added, st.growth_rows_copied), g0))
              for st, g0 in zip(state.sdm_states, growth0)]
    return dict(total_ms=sum(life_ms) + sum(dec_ms), decode_ms=sum(dec_ms), lifecycle_ms=sum(life_ms),
                clocks=clocks.summary(), setup_s=setup_s, stats=stats, quantum=quantum,
                growth_events=sum(g[0] for g in growth), growth_rows_added=sum(g[1] for g in growth),
                growth_rows_copied=sum(g[2] for g in growth),
                allocated_rows=sum(int(st.allocated_rows_tensor()) for st in state.sdm_states),
                capacity_rows=sum(st.capacity_rows for st in state.sdm_states),
                storage=state.storage_bytes(), banks=banks, live=live)


def cpu_churn_rate(seconds: float, quantum_steps: int) -> dict:
    """The oracle's churn loop on 8 live slots (32 banks) of one layer: decode
    steps with release -> retain -> sparse-prefill cohort -> append on
    completion, extrapolated to 256 slots x 7 layers per step (banks are
    independent, so CPU time scales with their number)."""
    from oracle import cow_oracle as O

    rng = np.random.default_rng(12)
    live = 8
    banks = live * CH_HEADS
    q = O.growth_quantum_rows(banks, WRITES, quantum_steps)
    m0 = (0.02 * rng.standard_normal((CH_HEADS, CH_SLOTS, WIDTH))).astype(np.float32)

    def prefill(requests, tokens):
        b = requests * CH_HEADS
        routes = lambda k: np.stack([O.uniform_routes(rng, b, CH_SLOTS, k) for _ in range(tokens)], 1)
        st, _ = O.sparse_prefill(
            m0, np.tile(np.arange(CH_HEADS), requests), routes(WRITES),
            O.softmax(rng.standard_normal((b, tokens, WRITES), dtype=np.float32)),
            rng.standard_normal((b, tokens, WIDTH), dtype=np.float32), rng.random((b, tokens), dtype=np.float32),
            -rng.random((b, tokens), dtype=np.float32), routes(READS),
            O.softmax(rng.standard_normal((b, tokens, READS), dtype=np.float32)), growth_quantum_rows=q)
        return st

    st = prefill(live, CH_WARM_PREFIX // 16)
    remaining = rng.integers(1, CH_MAX_LEN + 1, size=live)
    xs = [O.synthetic_step_inputs(rng, banks, CH_SLOTS, WIDTH, WRITES, READS) for _ in range(4)]
    n = completions = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        done = np.nonzero(remaining == 0)[0]
        if done.size:
            completions += done.size
            released = (done[:, None] * CH_HEADS + np.arange(CH_HEADS)).reshape(-1)
            O.release(st, released)
            O.retain_banks(st, np.setdiff1d(np.arange(st.banks), released))
            O.append_banks_from(st, prefill(int(done.size), CH_PROMPT))
            remaining = np.concatenate([remaining[remaining > 0],
                                        rng.integers(CH_MIN_LEN, CH_MAX_LEN + 1, size=done.size)])
        O.prepare_step_capacity(st, banks * WRITES)
        O.packed_step(st, **xs[n % len(xs)])
        remaining = remaining - 1
        n += 1
    dt = time.perf_counter() - t0
    step_s = dt / n * (CH_LIVE / live) * LAYERS
    return {"value": CH_LIVE / step_s, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n} oracle churn steps of {banks} banks (8 live slots x 4 heads, N={CH_SLOTS}), "
                      f"{completions} completions with release/retain/prefill/append, one layer, {dt:.1f} s, "
                      f"extrapolated to {CH_LIVE} slots x {LAYERS} layers per step"}


# --------------------------------------------------------------------------
# Configuration 2: whole-model decode
# --------------------------------------------------------------------------

M_VOCAB, M_MAXLEN, M_LAYOUT, M_WIDTH, M_HEADS, M_BATCH, M_PREFIX = 50257, 512, "BBBBBBBA", 128, 4, 16, 256


def run_gpu_model(args, rank, world, device):
    """Random-init 8-layer model (7 SDM layers + 1 attention layer), batch 16 per
    GPU, prefix 256 through the prefill handoff, then ``LanguageModel.decode``
    steps on seeded synthetic token ids.  Every timed step is one public
    decode token of the whole model (controller, fused packed step per SDM
    layer, K/V-cache attention, MLPs, vocabulary head), replayed as one CUDA
    graph by ``GraphedDecode``; the eager ``LanguageModel.decode`` is timed
    beside it.  The e2e leg also copies the step's ids from pinned host memory
    and reads the greedy next ids back."""
    from copy_on_write_sdm_b200.graph import GraphedDecode
    from copy_on_write_sdm_b200.model import LanguageModel

    K, Wm = args.steps, args.warmup
    if M_PREFIX + K + Wm > M_MAXLEN:
        raise SystemExit(f"model workload: prefix {M_PREFIX} + steps + warmup must fit {M_MAXLEN} positions")
    torch.manual_seed(0)
    model = LanguageModel(vocab_size=M_VOCAB, maximum_sequence_length=M_MAXLEN, layout=M_LAYOUT, width=M_WIDTH,
                          heads=M_HEADS, slots=SLOTS, reads=READS, writes=WRITES, memory_heads=HEADS,
                          activation_dtype=torch.float32)
    model.initialize_role_keyed(0)
    model = model.to(device).eval()
    gen = torch.Generator().manual_seed(100 + rank)
    ids = torch.randint(0, M_VOCAB, (M_BATCH, M_PREFIX + 2 * (K + Wm)), generator=gen)
    ids_dev = ids.to(device)
    t0 = time.time()
    _, state = model.prefill(ids_dev[:, :M_PREFIX], capacity=M_MAXLEN)
    torch.cuda.synchronize(device)
    setup_s = time.time() - t0
    stream = torch.cuda.current_stream(device)
    pos = M_PREFIX
    for _ in range(Wm):
        model.decode(ids_dev[:, pos:pos + 1], state)
        pos += 1
    torch.cuda.synchronize(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    with ClockSampler(device.index) as clocks:
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        for i in range(K):
            ev[i][0].record(stream)
            model.decode(ids_dev[:, pos:pos + 1], state)
            ev[i][1].record(stream)
            pos += 1
        torch.cuda.synchronize(device)
    eager_ms = sum(a.elapsed_time(b) for a, b in ev)
    # The same steps by CUDA-graph replay (GraphedDecode) on a fresh prefill of the same prompts.
    _, state = model.prefill(ids_dev[:, :M_PREFIX], capacity=M_MAXLEN)
    runner = GraphedDecode(model, state)
    pos = M_PREFIX
    for _ in range(Wm):
        runner.step(ids_dev[:, pos:pos + 1])
        pos += 1
    torch.cuda.synchronize(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    with ClockSampler(device.index) as clocks:
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        for i in range(K):
            ev[i][0].record(stream)
            runner.step(ids_dev[:, pos:pos + 1])
            ev[i][1].record(stream)
            pos += 1
        torch.cuda.synchronize(device)
    dev_ms = sum(a.elapsed_time(b) for a, b in ev)
    # e2e: a fresh prefill, then K graphed steps fed from pinned host ids, greedy ids read back
    _, state = model.prefill(ids_dev[:, :M_PREFIX], capacity=M_MAXLEN)
    runner = GraphedDecode(model, state)
    # one contiguous pinned [B,1] block per step, as a serving loop holds the next ids
    host_ids = ids[:, M_PREFIX:].t().contiguous().unsqueeze(-1).pin_memory()
    nxt = torch.empty(M_BATCH, 1, dtype=torch.int64).pin_memory()
    for i in range(Wm):
        runner.step(host_ids[i].to(device, non_blocking=True))
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(Wm, Wm + K):
        logits = runner.step(host_ids[i].to(device, non_blocking=True))
        nxt.copy_(logits.argmax(-1), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    state_bytes = state.storage_bytes()
    return dict(total_ms=dev_ms, eager_ms=eager_ms, e2e_ms=e0.elapsed_time(e1), clocks=clocks.summary(),
                setup_s=setup_s, captures=runner.captures,
                state_bytes=state_bytes, h2d=host_ids[0].numel() * 8, d2h=nxt.numel() * 8)


def main_model(args, rank, world, device) -> int:
    from copy_on_write_sdm_b200.sharding import reduce_over_ranks

    res = run_gpu_model(args, rank, world, device)
    total_ms, e2e_ms, eager_ms = reduce_over_ranks([res["total_ms"], res["e2e_ms"], res["eager_ms"]], op="max",
                                                   device=device)
    if rank != 0:
        torch.distributed.destroy_process_group()
        return 0
    K = args.steps
    tokens = M_BATCH * world * K
    line = {
        "metric": METRIC, "value": tokens / (total_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic token ids, random-init weights (seed 0)",
        "config": {"workload": "config 2 whole-model decode: LanguageModel vocab 50257, max_len 512, layout "
                               "BBBBBBBA, width 128, 4 attention heads, SDM N=256 D=128 H=1 top-16/top-4, "
                               "FP32 activations and SDM state",
                   "batch_per_gpu": M_BATCH, "global_batch": M_BATCH * world, "prefix": M_PREFIX,
                   "parallelism": f"requests sharded, {M_BATCH} per GPU x {world} GPU(s), no collective",
                   "l2": "model and state (~60 MB) stay L2-resident; steps timed back to back"},
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": res["h2d"],
                "d2h_bytes_per_step": res["d2h"],
                "path": "GraphedDecode.step per step with ids copied from pinned host memory and the greedy "
                        "next ids copied back"},
        "eager": {"value": tokens / (eager_ms / 1e3), "unit": "tokens/s", "ms_per_step": eager_ms / K,
                  "path": "LanguageModel.decode (the reference's eager call sequence)"},
        "graph_captures": res["captures"],
        "gpu_launches": (3 * 7 + 1) * K,
        "gpu_launches_note": "per step: for each of the 7 SDM layers cow_controller_kernel, the fused decode "
                             "step and cow_readout_kernel (readout + residual + MLP), and one "
                             "cow_attention_kernel for the dense block; the embedding, final norm and "
                             "vocabulary head run as PyTorch kernels",
        "clocks": res["clocks"],
        "cpu_baseline": None,
        "cpu_baseline_note": "the CPU port covers the SDM step and allocator, not the whole model",
        "retained_state": res["state_bytes"], "setup_s": res["setup_s"],
    }
    emit(line)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


# --------------------------------------------------------------------------
# CPU arms (the reference's algorithm, restated in oracle/)
# --------------------------------------------------------------------------


def cpu_decode_rate(seconds: float, threads: int, *, warmup: int = 0, steps: int | None = None) -> dict:
    """Tokens/s of the oracle's packed decode step on this host (bounded sample).

    The sample starts from a post-prefix pool (every slot private, as uniform
    2,048-token prefixes leave it), 7 layers x 64 requests, and runs decode
    steps -- ``steps`` of them after ``warmup``, or as many as fit in
    ``seconds`` -- with the layers spread over ``threads`` host threads.
    """
    from oracle import cow_oracle as O

    rng = np.random.default_rng(7)
    banks = BATCH * HEADS
    pools = []
    for _ in range(LAYERS):
        m0 = (0.02 * rng.standard_normal((HEADS, SLOTS, WIDTH))).astype(np.float32)
        dense = rng.standard_normal((banks, SLOTS, WIDTH)).astype(np.float32)
        pools.append(O.from_dense_overlay(m0, dense, np.ones((banks, SLOTS), bool),
                                          template_indices=np.zeros(banks, np.int64),
                                          capacity_rows=banks * SLOTS))
    batches = [[O.synthetic_step_inputs(rng, banks, SLOTS, WIDTH, WRITES, READS) for _ in range(LAYERS)]
               for _ in range(8)]
    done = 0
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        def one(i):
            list(ex.map(lambda lx: O.packed_step(lx[0], **lx[1]), zip(pools, batches[i % len(batches)])))

        for i in range(warmup):
            one(i)
        t0 = time.perf_counter()
        while (steps is not None and done < steps) or (steps is None and time.perf_counter() - t0 < seconds):
            one(done)
            done += 1
        dt = time.perf_counter() - t0
    return {"value": BATCH * done / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{done} decode steps x {LAYERS} layers x {banks} banks (N={SLOTS}, D={WIDTH}, "
                      f"top-{READS}/top-{WRITES}) from a post-prefix pool, {dt:.2f} s, numpy oracle"}


def _hbm_peak():
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peaks_path):
        return json.load(open(peaks_path))["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def _reduce_dict(d: dict, device) -> dict:
    """Sum of a dict of byte counts over ranks (the dict itself at one rank)."""
    from copy_on_write_sdm_b200.sharding import reduce_over_ranks

    keys = sorted(d)
    vals = reduce_over_ranks([float(d[k]) for k in keys], op="sum", device=device)
    return {k: int(v) for k, v in zip(keys, vals)}


def config_block(world: int) -> dict:
    return {"workload": "config 3 synthetic random-route serving screen: 7 independent SDM pools, N=256, D=128, "
                        "H=1, top-16 read/top-4 write, uniform seeded routes, prefix 2048 (sparse prefill), "
                        "growth quantum 4 steps",
            "batch_per_gpu": BATCH, "global_batch": BATCH * world, "prefix": PREFIX,
            "layers": LAYERS, "slots": SLOTS, "width": WIDTH, "heads": HEADS, "reads": READS, "writes": WRITES,
            "growth_quantum_rows": max(16, BATCH * HEADS * WRITES * QUANTUM_STEPS),
            "parallelism": f"requests sharded, {BATCH} per GPU x {world} GPU(s), no collective",
            "l2": f"inputs larger than L2: the K timed steps run in one CUDA graph between one device event "
                  f"pair, step i on replica i mod {REPLICAS} of this GPU's pools (independent copies taken after "
                  f"the warm-up), so the other replicas' steps move more than twice the 126 MB L2 between two "
                  f"visits of a replica; 'flushed_event_timed' keeps the earlier discipline (256 MiB L2 flush "
                  f"and an event pair around every step, on the pools themselves)",
            "capacity_proof": "timed device steps and end-to-end steps are proven up front "
                              "(prepare_step_capacity for all of them before timing); the per-step proof still "
                              "runs in every end-to-end step"}


_RESULT_OUT = None


def emit(line: dict) -> None:
    """Write the one result line to the process's original stdout."""
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def _reserve_stdout() -> None:
    """Keep the original stdout for the result line and send everything else that
    writes to file descriptor 1 (library banners, NCCL) to stderr."""
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def _e2e_block(tokens, res, e2e_ms, e2e_mapped_ms) -> dict:
    """End-to-end line: the faster of the two host-to-host runtime paths (both
    move the same bytes over PCIe every step), the other and the one-step-at-a-
    time path beside it."""
    piped = {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
             "path": "DecodeSession.step_host_pipelined: one pinned H2D copy, capacity proof + one fused launch, "
                     "one D2H copy; the copies of neighbouring steps overlap the decode on two side streams",
             "host_us_per_step": res.get("piped_host_us"),
             "note": "host_us_per_step: host time of the step_host_pipelined calls in the timed loop; a step "
                     "longer than that waits on the PCIe copies (340 KB in, 229 KB out per step)"}
    mapped = {"value": tokens / (e2e_mapped_ms / 1e3), "unit": "tokens/s",
              "path": "DecodeSession.step_host_mapped: capacity proof + one fused launch whose kernel reads the "
                      "step's pinned host bytes over PCIe and writes the readouts to pinned host memory (zero-copy)",
              "breakdown": res["mapped_device"]}
    best, other, name = (piped, mapped, "mapped") if piped["value"] >= mapped["value"] else (mapped, piped, "pipelined")
    return {**best, "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"], name: other,
            "serial": {"value": tokens / (res["e2e_serial_ms"] / 1e3), "unit": "tokens/s",
                       "path": "DecodeSession.step_host: copy, decode and read back one step at a time"}}


def _leg_line(res, total_ms, K, batch_per_gpu, world, note) -> dict:
    """Summary of a flushed-trace sub-leg (rank 0's own figures beside the max over ranks)."""
    peak, peak_src = _hbm_peak()
    per_launch = algorithmic_bytes(res["banks"] * LAYERS, res["first_touches"] // max(K, 1))
    mean_s = res["total_ms"] / K / 1e3
    out = {"value": batch_per_gpu * world * K / (total_ms / 1e3), "unit": "tokens/s", "ms_per_step": total_ms / K,
           "batch_per_gpu": batch_per_gpu, "global_batch": batch_per_gpu * world, "note": note,
           "first_touches_in_timed_steps": res["first_touches"],
           "roofline": {"bound": "hbm", "achieved": per_launch / mean_s / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": per_launch / mean_s / 1e9 / peak, "peak_source": peak_src,
                        "algorithmic_bytes_per_launch": per_launch, "mean_launch_us": mean_s * 1e6},
           "retained_state": res["state_bytes"], "clocks": res["clocks"]}
    out["flushed_event_timed"] = {"ms_per_step": res["flushed_ms"] / K,
                                  "first_touches_in_timed_steps": res["flushed_first_touches"]}
    if res.get("dense_ms") is not None:
        out["dense_control"] = {"ms_per_step": res["dense_ms"] / K,
                                "packed_latency_overhead_pct": 100.0 * (res["flushed_ms"] / res["dense_ms"] - 1.0),
                                "note": "both flushed and event-timed per step"}
    inc = res.get("incremental")
    if inc is not None:
        out["graph_incremental"] = {**inc, "packed_latency_overhead_pct": 100.0 * (inc["packed_us"] / inc["dense_us"] - 1.0)}
    return out


def sub_legs(args, rank, world, device, res, total_ms) -> dict:
    """Legs of the default run beside the headline (all ranks take part; rank 0 reports).

    * ``allocating_prefix16``: the screen at prefix 16, the reference's own
      serving-screen prefix, where timed steps pop rows (about half of the
      routed slots are still shared), with its dense control;
    * ``strong_split``: B=64 requests in total, 64/N per GPU (N > 1);
    * ``scaleout``: configuration 4 (1,024 requests over all GPUs, prefix
      4,096, Zipf routes), steps capped at 32."""
    from copy_on_write_sdm_b200.sharding import reduce_over_ranks

    K = args.steps
    legs = {}
    if not args.legs:
        return legs
    r16 = run_gpu(args, rank, world, device, prefix=16, extras=False)
    (t16,) = reduce_over_ranks([r16["total_ms"]], op="max", device=device)
    legs["allocating_prefix16"] = _leg_line(r16, t16, K, BATCH, world,
                                            "configuration 3 at prefix 16 (reference serving screen, "
                                            "benchmark_serving.py:628): timed steps allocate rows")
    if world > 1:
        rs = run_gpu(args, rank, world, device, batch=max(1, BATCH // world), extras=False)
        (ts,) = reduce_over_ranks([rs["total_ms"]], op="max", device=device)
        legs["strong_split"] = {**_leg_line(rs, ts, K, max(1, BATCH // world), world,
                                            f"B={BATCH} requests in total, {BATCH // world} per GPU"),
                                "scaling": "strong"}
    else:
        legs["strong_split"] = {"value": BATCH * K / (total_ms / 1e3), "unit": "tokens/s", "scaling": "strong",
                                "note": "at one GPU the strong split is the headline itself"}
    torch.cuda.empty_cache()
    so_args = argparse.Namespace(**vars(args))
    so_args.steps, so_args.warmup = min(args.steps, 32), min(args.warmup, 4)
    so_args.requests, so_args.prefix = SO_REQUESTS, SO_PREFIX
    so_args.hash_leg = True
    so = scaleout_line(so_args, rank, world, device, cpu_seconds=min(args.cpu_seconds, 5.0))
    torch.cuda.empty_cache()
    if so is not None:
        legs["scaleout"] = {k: so.get(k) for k in ("value", "unit", "ms_per_step", "steps", "scaling", "roofline",
                                                "cpu_baseline", "retained_state", "first_touches_in_timed_steps",
                                                "mean_touched_rows_per_bank", "clocks", "config", "setup_s",
                                                "hashed_map")}
    return legs


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--workload", default="screen", choices=["screen", "model", "scaleout", "churn"],
                    help="screen: configuration 3 (default, the headline); model: configuration 2; "
                         "scaleout: configuration 4; churn: configuration 5")
    ap.add_argument("--requests", type=int, default=SO_REQUESTS, help="scaleout: requests over all GPUs")
    ap.add_argument("--prefix", type=int, default=SO_PREFIX, help="scaleout: prefix tokens")
    ap.add_argument("--hash-leg", action="store_true", help="scaleout: also time the pools on hashed maps")
    ap.add_argument("--hash-max-load", type=float, default=0.0,
                    help="scaleout: largest fill of a bank's hashed table (default: the library's 0.7)")
    ap.add_argument("--quantum-steps", type=int, default=4, help="churn: growth quantum in decode steps")
    ap.add_argument("--trim-every", type=int, default=0, help="churn: trim the pools every this many steps")
    ap.add_argument("--churn-admit", default="prefix", choices=["prefix", "prefill"],
                    help="churn: admit cohorts by prefilling straight into the live pools (admit_prefix) or by "
                         "prefilling pools of their own and admitting those (prefill + admit)")
    ap.add_argument("--no-legs", dest="legs", action="store_false",
                    help="screen: skip the prefix-16, strong-split and configuration-4 legs")
    ap.add_argument("--churn-warm-prefix", type=int, default=CH_WARM_PREFIX,
                    help="churn: prefix tokens of the initial batch")
    args = ap.parse_args()
    _reserve_stdout()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        threads = min(LAYERS, os.cpu_count() or 1)
        cpu = cpu_decode_rate(0.0, threads, warmup=args.warmup, steps=args.steps)
        v = cpu["value"]
        line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * BATCH / v,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config_block(args.gpus), "cpu_baseline": cpu,
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        emit(line)
        return 0

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        # NCCL's own output (version banner, NCCL_DEBUG lines) reaches stderr:
        # _reserve_stdout keeps the result line alone on stdout.
        torch.distributed.init_process_group("nccl", device_id=device)
    torch.backends.cuda.matmul.allow_tf32 = False
    if args.workload == "scaleout":
        return main_scaleout(args, rank, world, device)
    if args.workload == "churn":
        return main_churn(args, rank, world, device)
    if args.workload == "model":
        return main_model(args, rank, world, device)
    res = run_gpu(args, rank, world, device)

    from copy_on_write_sdm_b200.sharding import reduce_over_ranks

    # Job time = the slowest rank (each rank owns its own 64 requests).
    total_ms, e2e_ms, e2e_mapped_ms = reduce_over_ranks([res["total_ms"], res["e2e_ms"], res["e2e_mapped_ms"]],
                                                        op="max", device=device)
    state_all = _reduce_dict(res["state_bytes"], device)
    legs = sub_legs(args, rank, world, device, res, total_ms)
    if rank != 0:
        torch.distributed.destroy_process_group()
        return 0

    K = args.steps
    tokens = BATCH * world * K
    value = tokens / (total_ms / 1e3)
    peak, peak_src = _hbm_peak()
    per_launch = algorithmic_bytes(BATCH * HEADS * LAYERS, res["first_touches"] // max(K, 1))
    mean_launch_s = (res["total_ms"] / K) / 1e3
    achieved = per_launch / mean_launch_s / 1e9
    dense_bytes = dense_algorithmic_bytes(BATCH * HEADS * LAYERS)
    cpu = cpu_decode_rate(args.cpu_seconds, min(LAYERS, os.cpu_count() or 1))
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_block(world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": TRAFFIC_SCREEN["bytes_per_launch"],
                     "traffic_source": TRAFFIC_SCREEN["source"], "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": per_launch, "mean_launch_us": mean_launch_s * 1e6,
                     "kernel": "cow_decode_split_kernel"},
        "e2e": _e2e_block(tokens, res, e2e_ms, e2e_mapped_ms),
        "gpu_launches": K,
        "graph_incremental": None if res["incremental"] is None else {
            **res["incremental"],
            "packed_latency_overhead_pct": 100.0 * (res["incremental"]["packed_us"] / res["incremental"]["dense_us"] - 1.0),
            "note": "cold step's added device time in a graph of K x (L2 flush, step) minus K x flush"},
        "eager_flushed": res["eager"],
        "single_launch": {"value": BATCH / (res["single_ms"] / 1e3), "unit": "tokens/s",
                          "ms_per_step": res["single_ms"],
                          "note": "one step per graph launch, timed alone (median); includes host submission"},
        "clocks": res["clocks"],
        "cpu_baseline": cpu,
        "flushed_event_timed": {
            "value": BATCH * K / (res["flushed_ms"] / 1e3), "unit": "tokens/s", "ms_per_step": res["flushed_ms"] / K,
            "first_touches_in_timed_steps": res["flushed_first_touches"],
            "note": "the same K steps on the pools themselves, each in one CUDA graph after a 256 MiB L2 flush "
                    "between its own event pair (the pair adds ~4.5 us of graph scheduling to each interval)"},
        "dense_control": None if res["dense_ms"] is None else {
            "value": BATCH * K / (res["dense_ms"] / 1e3), "unit": "tokens/s",
            "ms_per_step": res["dense_ms"] / K,
            "packed_latency_overhead_pct": 100.0 * (res["flushed_ms"] / res["dense_ms"] - 1.0),
            "achieved_gbs": dense_bytes / (res["dense_ms"] / K / 1e3) / 1e9,
            "note": "dense table and packed step both flushed and event-timed per step"},
        "warm_l2_trace": None if res["warm_ms"] is None else {
            "value": BATCH * K / (res["warm_ms"] / 1e3), "unit": "tokens/s", "ms_per_step": res["warm_ms"] / K,
            "dense_ms_per_step": res["dense_warm_ms"] / K,
            "packed_latency_overhead_pct": 100.0 * (res["warm_ms"] / res["dense_warm_ms"] - 1.0),
            "note": "all K steps in one CUDA graph, back to back, pool state L2-resident"},
        "retained_state": {"allocated_rows": res["allocated_rows"], "capacity_rows": res["capacity_rows"],
                           "live_value_bytes": res["live_value_bytes"], **res["state_bytes"],
                           "all_gpus": state_all},
        "first_touches_in_timed_steps": res["first_touches"],
        "setup_s": res["setup_s"],
        **legs,
    }
    emit(line)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def scaleout_line(args, rank, world, device, *, cpu_seconds) -> dict | None:
    """Configuration 4 (strong scaling: ``args.requests`` over all ranks); rank 0
    returns the result line, the other ranks None."""
    from copy_on_write_sdm_b200.sharding import reduce_over_ranks

    res = run_gpu_scaleout(args, rank, world, device)
    total_ms = reduce_over_ranks([res["total_ms"]], op="max", device=device)[0]
    state_bytes = _reduce_dict(res["state_bytes"], device)
    if rank != 0:
        return None
    K = args.steps
    tokens = res["requests"] * world * K
    peak, peak_src = _hbm_peak()
    per_launch = algorithmic_bytes(res["banks"] * LAYERS, res["first_touches"] // max(K, 1))
    mean_s = res["total_ms"] / K / 1e3
    achieved = per_launch / mean_s / 1e9
    line = {
        "metric": METRIC, "value": tokens / (total_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config 4 large-address-space scale-out: 7 SDM pools, N=65536, D=128, H=8, "
                               "top-16/top-4, Zipf(1.1) routes over a seeded address permutation",
                   "global_batch": args.requests, "requests_per_gpu": res["requests"], "prefix": args.prefix,
                   "parallelism": f"requests sharded over {world} GPU(s), no collective",
                   "prefix_state": "written-address union of the Zipf prefix packed in nonzero() order, rows from M0",
                   "l2": "pool state (>100 GB at 1 GPU) far exceeds L2; steps timed back to back"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": TRAFFIC_SCALEOUT["bytes_per_launch_per_bank"] * res["banks"] * LAYERS,
                     "traffic_source": TRAFFIC_SCALEOUT["source"], "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": per_launch,
                     "mean_launch_us": mean_s * 1e6, "kernel": "cow_count_kernel + cow_decode_kernel<f32,1,4,1>",
                     "timing": "rank 0's launches, each timed by its own CUDA event pair on the launching stream"},
        "gpu_launches": 2 * K, "clocks": res["clocks"],
        "cpu_baseline": cpu_scaleout_rate(cpu_seconds, res["requests"] * world, args.prefix),
        "mean_touched_rows_per_bank": res["mean_touched_rows_per_bank"],
        "first_touches_in_timed_steps": res["first_touches"],
        "retained_state": {"all_gpus": state_bytes, "rank0": res["state_bytes"]},
        "setup_s": res["setup_s"],
    }
    h = res.get("hashed")
    if h is not None:
        hb = algorithmic_bytes(res["banks"] * LAYERS, h["first_touches"] // max(K, 1))
        hs = h["total_ms"] / K / 1e3
        line["hashed_map"] = {
            "value": res["requests"] * K / (h["total_ms"] / 1e3), "unit": "tokens/s", "ms_per_step": h["total_ms"] / K,
            "roofline": {"achieved": hb / hs / 1e9, "peak": peak, "frac": hb / hs / 1e9 / peak, "unit": "GB/s",
                         "note": "algorithmic bytes as for the dense map (map lookups counted at 4 B)"},
            "map_bytes_rank0": h["map_bytes"], "dense_map_bytes_rank0": h["dense_map_bytes"],
            "table_slots_per_bank": h["table_slots"], "first_touches_in_timed_steps": h["first_touches"],
            "status": h["status"],
            "note": "rank 0: the same pools converted to per-bank hashed tables, next K steps of the same trace"}
    return line


def main_scaleout(args, rank, world, device) -> int:
    line = scaleout_line(args, rank, world, device, cpu_seconds=args.cpu_seconds)
    if line is not None:
        line["e2e"] = None
        emit(line)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def main_churn(args, rank, world, device) -> int:
    from copy_on_write_sdm_b200.sharding import reduce_over_ranks

    res = run_gpu_churn(args, rank, world, device)
    (total_ms,) = reduce_over_ranks([res["total_ms"]], op="max", device=device)
    if rank != 0:
        torch.distributed.destroy_process_group()
        return 0
    K = args.steps
    tokens = res["live"] * world * K
    line = {
        "metric": METRIC, "value": tokens / (total_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config 5 continuous-batching churn: 7 SDM pools, N=4096, D=128, H=4, top-16/top-4, "
                               "256 live slots, Poisson(8) arrivals, lengths U[64,4096], 64-token prompts "
                               "(sparse prefill), release -> compact -> admit on completion",
                   "live_slots_per_gpu": res["live"], "global_batch": res["live"] * world,
                   "growth_quantum_steps": args.quantum_steps, "growth_quantum_rows": res["quantum"],
                   "trim_every": args.trim_every, "initial_prefix": args.churn_warm_prefix,
                   "admission": ("admit_prefix: cohorts prefilled straight into the live pools" if args.churn_admit
                                 == "prefix" else "prefill pools of their own, then admit"),
                   "parallelism": f"requests sharded, {res['live']} slots per GPU x {world} GPU(s), no collective",
                   "l2": "pool state (>10 GB) exceeds L2; steps timed back to back"},
        "decode_ms_per_step": res["decode_ms"] / K, "lifecycle_ms_per_step": res["lifecycle_ms"] / K,
        "lifecycle": {**res["stats"], "growth_events": res["growth_events"],
                      "growth_rows_added": res["growth_rows_added"], "growth_rows_copied": res["growth_rows_copied"]},
        "retained_state": {"allocated_rows": res["allocated_rows"], "capacity_rows": res["capacity_rows"],
                           **res["storage"]},
        "e2e": None, "gpu_launches": K,
        "gpu_launches_note": "fused decode launches; lifecycle kernels (release, retain, prefill, append, grow) "
                             "vary with completions and are not counted",
        "clocks": res["clocks"],
        "cpu_baseline": cpu_churn_rate(args.cpu_seconds, args.quantum_steps),
        "setup_s": res["setup_s"],
    }
    emit(line)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
