"""SDM controller (PyTorch) feeding the packed copy-on-write kernels.

The controller is the caller of the hot path, not the hot path: layer norm,
product-key top-k routing, value / gate projections before the step, readings
norm + output gate + projection after it (reference ``copy_on_write_sdm/sdm.py:
96-159, 998-1262``; decode split at ``inference.py:459-535``).  Parameter names
and shapes equal the reference's ``SparseDeltaMemory`` so its checkpoints load
unchanged (``load_state_dict``).

The dense training recurrence (and its backward) is not part of this package:
the eval ``forward`` runs the exact recurrence through the sparse prefill
kernel on a throw-away pool, so it never materialises ``[B,T,N,D]`` states.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from .allocator import PackedSDMCopyOnWriteState


def product_key_routes(projected: torch.Tensor, *, slots: int, selected: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Product-key address selection (reference sdm.py:96-159).

    ``projected [..., 2*sqrt(N)]`` holds two codebook score vectors.  Each
    codebook keeps its best ``min(k, sqrt(N))`` entries, the Cartesian sums of
    the two shortlists are ranked, the best ``k`` pairs give addresses
    ``first * sqrt(N) + second``, addresses are sorted ascending and the
    matching pair scores are softmax-normalised.  Returns ``(weights, indices)``.
    """

    if projected.ndim != 3:
        raise ValueError("product-key projection must be [B,T,2*sqrt(N)]")
    root = math.isqrt(slots)
    if root * root != slots or projected.shape[-1] != 2 * root:
        raise ValueError("slot count and product-key projection do not match")
    if not 1 <= selected <= slots:
        raise ValueError("selected product keys must be between one and slots")
    short = min(selected, root)
    a_score, a_idx = torch.topk(projected[..., :root], k=short, dim=-1)
    b_score, b_idx = torch.topk(projected[..., root:], k=short, dim=-1)
    # pair (i, j) -> flat position i * short + j, score a_i + b_j
    pair_score = (a_score[..., :, None] + b_score[..., None, :]).flatten(-2)
    pair_addr = (a_idx[..., :, None] * root + b_idx[..., None, :]).flatten(-2)
    best_score, best_pos = torch.topk(pair_score, k=min(selected, pair_score.shape[-1]), dim=-1)
    addr = pair_addr.gather(-1, best_pos)
    addr, order = addr.sort(dim=-1)
    return torch.softmax(best_score.gather(-1, order), dim=-1), addr


@dataclass(frozen=True)
class SDMStepInputs:
    """Controller outputs for ``T`` positions, laid out per bank (``b*H + h``)."""

    normalized: torch.Tensor  # [B, T, width]
    write_indices: torch.Tensor  # [B*H, T, W]
    write_weights: torch.Tensor
    values: torch.Tensor  # [B*H, T, head_width]
    input_gate: torch.Tensor  # [B*H, T]
    forget_log_gate: torch.Tensor
    read_indices: torch.Tensor  # [B*H, T, R]
    read_weights: torch.Tensor


class SparseDeltaMemory(nn.Module):
    """One physical SDM layer's controller (reference sdm.py:998-1262 parameter layout)."""

    def __init__(self, width: int, *, slots: int, reads: int, writes: int, memory_heads: int = 1,
                 norm_eps: float = 1e-6) -> None:
        super().__init__()
        if width <= 0 or slots <= 0 or memory_heads <= 0:
            raise ValueError("width, slots, and memory_heads must be positive")
        if width % memory_heads:
            raise ValueError("width must be divisible by memory_heads")
        root = math.isqrt(slots)
        if root * root != slots:
            raise ValueError("faithful SDM slots must be a perfect square")
        if not 1 <= reads <= slots or not 1 <= writes <= slots:
            raise ValueError("read and write counts must lie within the table")
        self.width, self.slots, self.total_slots = width, slots, slots
        self.reads, self.writes, self.memory_heads = reads, writes, memory_heads
        self.head_width = width // memory_heads
        self.key_width_per_head = 2 * root
        self.key_width = memory_heads * self.key_width_per_head
        self.input_norm = nn.LayerNorm(width)
        self.read_projection = nn.Linear(width, self.key_width)
        self.write_projection = nn.Linear(width, self.key_width)
        self.value_projection = nn.Linear(width, width)
        self.forget_projection = nn.Linear(width, memory_heads)
        self.input_projection = nn.Linear(width, memory_heads)
        self.A_log = nn.Parameter(torch.empty(memory_heads))
        self.dt_bias = nn.Parameter(torch.empty(memory_heads))
        self.output_gate = nn.Linear(width, width)
        self.output_projection = nn.Linear(width, width)
        self.initial_memory = nn.Parameter(torch.empty(memory_heads, slots, self.head_width))
        self.readings_norm = nn.LayerNorm(self.head_width, eps=norm_eps)
        self.reset_parameters()

    def _projections(self):
        return (self.read_projection, self.write_projection, self.value_projection, self.forget_projection,
                self.input_projection, self.output_gate, self.output_projection)

    def _init_gates(self) -> None:
        # A = U(0,16) clamped at 1e-4, stored as log; dt = exp(U(log 1e-3, log 1e-1)),
        # stored through the inverse softplus (Mamba-style initialisation).
        with torch.no_grad():
            self.A_log.copy_(torch.empty_like(self.A_log).uniform_(0.0, 16.0).clamp_(min=1e-4).log())
            dt = torch.empty_like(self.dt_bias).uniform_(math.log(1e-3), math.log(1e-1)).exp()
            self.dt_bias.copy_(dt + torch.log(-torch.expm1(-dt)))

    def reset_parameters(self) -> None:
        std = self.width ** -0.5
        for proj in self._projections():
            nn.init.trunc_normal_(proj.weight, mean=0.0, std=std, a=-3 * std, b=3 * std)
            nn.init.zeros_(proj.bias)
        self.input_norm.reset_parameters()
        self.readings_norm.reset_parameters()
        self._init_gates()
        nn.init.trunc_normal_(self.initial_memory, mean=0.0, std=std, a=-3 * std, b=3 * std)

    def reset_role_keyed(self, seed: int) -> None:
        """Seeded initialisation, one stream per parameter role (random-init serving runs)."""
        gen_state = torch.random.get_rng_state()
        try:
            std = self.width ** -0.5
            self.input_norm.reset_parameters()
            self.readings_norm.reset_parameters()
            for offset, proj in enumerate(self._projections(), start=1):
                torch.manual_seed(seed + offset)
                nn.init.trunc_normal_(proj.weight, mean=0.0, std=std, a=-3 * std, b=3 * std)
                nn.init.zeros_(proj.bias)
            torch.manual_seed(seed + 8)
            self._init_gates()
            torch.manual_seed(seed + 10)
            nn.init.trunc_normal_(self.initial_memory, mean=0.0, std=std, a=-3 * std, b=3 * std)
        finally:
            torch.random.set_rng_state(gen_state)

    # ---------------- controller ----------------

    def _per_bank(self, x: torch.Tensor, batch: int, time: int) -> torch.Tensor:
        """[B, T, H*k] -> [B*H, T, k] (bank = b*H + h)."""
        return x.reshape(batch, time, self.memory_heads, -1).permute(0, 2, 1, 3).reshape(
            batch * self.memory_heads, time, -1)

    def controller(self, tokens: torch.Tensor) -> SDMStepInputs:
        """Position-parallel routes, values and gates (reference inference.py:459-519, sdm.py:1149-1184)."""
        if tokens.ndim != 3 or tokens.shape[-1] != self.width:
            raise ValueError(f"SDM tokens must be [B,T,{self.width}]")
        batch, time, _ = tokens.shape
        if self._fused_routes_ok(tokens) and self._fused_controller_ok():
            return self._controller_step(tokens, batch, time)
        normalized = self.input_norm(tokens)
        if self._fused_routes_ok(tokens):
            return self._controller_fused(normalized, batch, time)
        read_w, read_i = product_key_routes(self._per_bank(self.read_projection(normalized), batch, time).reshape(
            batch * self.memory_heads, time, -1), slots=self.slots, selected=self.reads)
        write_w, write_i = product_key_routes(self._per_bank(self.write_projection(normalized), batch, time),
                                              slots=self.slots, selected=self.writes)
        values = self._per_bank(self.value_projection(normalized), batch, time)
        forget = -torch.exp(self.A_log) * F.softplus(self.forget_projection(normalized) + self.dt_bias)
        gate_in = torch.sigmoid(self.input_projection(normalized))
        return SDMStepInputs(
            normalized=normalized,
            write_indices=write_i, write_weights=write_w, values=values.contiguous(),
            input_gate=gate_in.permute(0, 2, 1).reshape(batch * self.memory_heads, time),
            forget_log_gate=forget.permute(0, 2, 1).reshape(batch * self.memory_heads, time),
            read_indices=read_i, read_weights=read_w,
        )

    def _fused_routes_ok(self, tokens: torch.Tensor) -> bool:
        root = math.isqrt(self.slots)
        return (tokens.is_cuda and tokens.dtype == torch.float32 and root <= 256 and self.reads <= 32
                and self.writes <= 32 and min(self.reads, root) <= 32 and min(self.writes, root) <= 32
                and all(p.dtype == torch.float32 for p in (self.A_log, self.dt_bias)))

    def _fused_controller_ok(self) -> bool:
        root = math.isqrt(self.slots)
        ntot = 4 * self.memory_heads * root + self.width + 2 * self.memory_heads
        norm = self.input_norm
        return (self.width <= 512 and ntot <= 4096 and norm.elementwise_affine and norm.weight is not None
                and norm.bias is not None and all(p.weight.dtype == torch.float32 for p in self._routing_linears()))

    def _routing_linears(self):
        return (self.read_projection, self.write_projection, self.value_projection, self.forget_projection,
                self.input_projection)

    def _stacked_weights(self):
        """[width, Ntot] transposed concatenation of the routing projections and their
        bias; rebuilt only when a parameter was replaced or changed in place."""
        params = [t for lin in self._routing_linears() for t in (lin.weight, lin.bias)]
        key = tuple((t.data_ptr(), t._version) for t in params)
        cached = self.__dict__.get("_stacked_cache")
        if cached is None or cached[0] != key:
            with torch.no_grad():
                wt = torch.cat([lin.weight for lin in self._routing_linears()], 0).t().contiguous()
                bias = torch.cat([lin.bias for lin in self._routing_linears()], 0).contiguous()
            cached = (key, wt, bias)
            self.__dict__["_stacked_cache"] = cached
        return cached[1], cached[2]

    def _controller_step(self, tokens: torch.Tensor, batch: int, time: int) -> SDMStepInputs:
        """The whole controller in one ``cow_controller_step`` launch (FP32): layer norm,
        the five routing projections, route selection, gates and value slices."""
        H = self.memory_heads
        device = tokens.device
        x = tokens.contiguous()
        wt, bias = self._stacked_weights()
        banks = batch * H
        normalized = torch.empty_like(x)
        read_i = torch.empty(banks, time, self.reads, dtype=torch.int64, device=device)
        read_w = torch.empty(banks, time, self.reads, dtype=torch.float32, device=device)
        write_i = torch.empty(banks, time, self.writes, dtype=torch.int64, device=device)
        write_w = torch.empty(banks, time, self.writes, dtype=torch.float32, device=device)
        values = torch.empty(banks, time, self.head_width, dtype=torch.float32, device=device)
        gate_in = torch.empty(banks, time, dtype=torch.float32, device=device)
        forget = torch.empty(banks, time, dtype=torch.float32, device=device)
        norm = self.input_norm
        _lib.check(_lib.load().cow_controller_step(
            x.data_ptr(), norm.weight.data_ptr(), norm.bias.data_ptr(), float(norm.eps), wt.data_ptr(),
            bias.data_ptr(), self.A_log.data_ptr(), self.dt_bias.data_ptr(), batch, time, self.width, H,
            math.isqrt(self.slots), self.reads, self.writes, normalized.data_ptr(), read_i.data_ptr(),
            read_w.data_ptr(), write_i.data_ptr(), write_w.data_ptr(), values.data_ptr(), gate_in.data_ptr(),
            forget.data_ptr(), _lib.stream_of(device)), "cow_controller_step")
        return SDMStepInputs(
            normalized=normalized, write_indices=write_i, write_weights=write_w, values=values,
            input_gate=gate_in, forget_log_gate=forget, read_indices=read_i, read_weights=read_w)

    def _controller_fused(self, normalized: torch.Tensor, batch: int, time: int) -> SDMStepInputs:
        """The same outputs as the PyTorch controller; the route selection and gates
        run as one ``cow_route_controller`` launch (FP32 activations)."""
        H = self.memory_heads
        device = normalized.device
        rp = self.read_projection(normalized).contiguous()
        wp = self.write_projection(normalized).contiguous()
        fp = self.forget_projection(normalized).contiguous()
        ip = self.input_projection(normalized).contiguous()
        a_log = self.A_log.detach().contiguous()
        dt_bias = self.dt_bias.detach().contiguous()
        banks = batch * H
        read_i = torch.empty(banks, time, self.reads, dtype=torch.int64, device=device)
        read_w = torch.empty(banks, time, self.reads, dtype=torch.float32, device=device)
        write_i = torch.empty(banks, time, self.writes, dtype=torch.int64, device=device)
        write_w = torch.empty(banks, time, self.writes, dtype=torch.float32, device=device)
        gate_in = torch.empty(banks, time, dtype=torch.float32, device=device)
        forget = torch.empty(banks, time, dtype=torch.float32, device=device)
        _lib.check(_lib.load().cow_route_controller(
            rp.data_ptr(), wp.data_ptr(), fp.data_ptr(), ip.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(),
            batch, time, H, math.isqrt(self.slots), self.reads, self.writes, read_i.data_ptr(), read_w.data_ptr(),
            write_i.data_ptr(), write_w.data_ptr(), gate_in.data_ptr(), forget.data_ptr(),
            _lib.stream_of(device)), "cow_route_controller")
        values = self._per_bank(self.value_projection(normalized), batch, time)
        return SDMStepInputs(
            normalized=normalized, write_indices=write_i, write_weights=write_w, values=values.contiguous(),
            input_gate=gate_in, forget_log_gate=forget, read_indices=read_i, read_weights=read_w)

    def finish(self, normalized: torch.Tensor, readings: torch.Tensor) -> torch.Tensor:
        """Readings norm, channel gate and output projection (reference inference.py:522-535)."""
        batch, time, _ = normalized.shape
        r = self.readings_norm(readings).reshape(batch, self.memory_heads, time, self.head_width)
        r = r.permute(0, 2, 1, 3).reshape(batch, time, self.width)
        return self.output_projection(torch.sigmoid(self.output_gate(normalized)) * r)

    def finish_residual(self, tokens: torch.Tensor, normalized: torch.Tensor, readings: torch.Tensor,
                        mlp: nn.Module) -> torch.Tensor:
        """``t = tokens + finish(normalized, readings)`` followed by ``t + mlp(t)``: the
        SDM layer's residual and the MLP block after it (reference inference.py:655-661).
        FP32 CUDA activations in eval mode run as one ``cow_readout_mlp_step`` launch."""
        if self._fused_readout_ok(tokens, normalized, readings, mlp):
            return self._readout_step(tokens, normalized, readings, mlp)
        tokens = tokens + self.finish(normalized, readings)
        return tokens + mlp(tokens)

    def _fused_readout_ok(self, tokens, normalized, readings, mlp) -> bool:
        rn, mn = self.readings_norm, getattr(mlp, "norm", None)
        if not (tokens.is_cuda and tokens.dtype == normalized.dtype == readings.dtype == torch.float32):
            return False
        if self.training or mlp.training or not isinstance(mn, nn.LayerNorm):
            return False
        act = getattr(mlp, "activation", None)
        if not (isinstance(act, nn.GELU) and act.approximate == "none"):
            return False
        if not (rn.elementwise_affine and rn.bias is not None and mn.elementwise_affine and mn.bias is not None):
            return False
        if self.output_gate.bias is None or self.output_projection.bias is None:
            return False
        if mlp.input.bias is not None or mlp.output.bias is not None:
            return False
        params = self._readout_params(mlp)
        # wider layers stream more weight per token than one block hides; PyTorch's
        # GEMMs are faster there (width 512: 51 us against 87 us for 16 tokens)
        return (self.width <= 256 and mlp.input.out_features <= 1024 and self.memory_heads <= 64
                and all(p.dtype == torch.float32 and p.is_cuda for p in params))

    def _readout_params(self, mlp):
        return (self.readings_norm.weight, self.readings_norm.bias, self.output_gate.weight, self.output_gate.bias,
                self.output_projection.weight, self.output_projection.bias, mlp.norm.weight, mlp.norm.bias,
                mlp.input.weight, mlp.output.weight)

    def _readout_weights(self, mlp):
        """Transposed ([in, out]) copies of the gate, output and MLP matrices; rebuilt
        only when a parameter was replaced or changed in place."""
        params = self._readout_params(mlp)
        key = (id(mlp),) + tuple((t.data_ptr(), t._version) for t in params)
        cached = self.__dict__.get("_readout_cache")
        if cached is None or cached[0] != key:
            with torch.no_grad():
                mats = tuple(w.t().contiguous() for w in (self.output_gate.weight, self.output_projection.weight,
                                                        mlp.input.weight, mlp.output.weight))
            cached = (key, mats)
            self.__dict__["_readout_cache"] = cached
        return cached[1]

    def _readout_step(self, tokens, normalized, readings, mlp) -> torch.Tensor:
        batch, time, _ = tokens.shape
        x, n = tokens.contiguous(), normalized.contiguous()
        r = readings.contiguous()
        if r.shape != (batch * self.memory_heads, time, self.head_width):
            raise ValueError("SDM readings must be [B*H,T,head_width]")
        wg, wo, w1, w2 = self._readout_weights(mlp)
        rn, mn = self.readings_norm, mlp.norm
        out = torch.empty_like(x)
        _lib.check(_lib.load().cow_readout_mlp_step(
            x.data_ptr(), n.data_ptr(), r.data_ptr(), rn.weight.data_ptr(), rn.bias.data_ptr(), float(rn.eps),
            wg.data_ptr(), self.output_gate.bias.data_ptr(), wo.data_ptr(), self.output_projection.bias.data_ptr(),
            mn.weight.data_ptr(), mn.bias.data_ptr(), float(mn.eps), w1.data_ptr(), w2.data_ptr(), batch, time,
            self.width, self.memory_heads, mlp.input.out_features, out.data_ptr(), _lib.stream_of(tokens.device)),
            "cow_readout_mlp_step")
        return out

    def template_indices(self, batch: int, device) -> torch.Tensor:
        return torch.arange(self.memory_heads, device=device, dtype=torch.int64).repeat(batch)

    def prefill(self, tokens: torch.Tensor, *, capacity_rows: int | None = None,
                maximum_future_allocations: int | None = None, growth_quantum_rows: int = 0,
                state_dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, PackedSDMCopyOnWriteState]:
        """Exact prefix pass + packed handoff through the sparse prefill kernel."""
        step = self.controller(tokens)
        batch = tokens.shape[0]
        state, readings = PackedSDMCopyOnWriteState.from_prefix_routes(
            self.initial_memory,
            step.write_indices, step.write_weights, step.values, step.input_gate, step.forget_log_gate,
            step.read_indices, step.read_weights,
            template_indices=self.template_indices(batch, tokens.device),
            capacity_rows=capacity_rows, state_dtype=state_dtype,
            maximum_future_allocations=maximum_future_allocations,
            growth_quantum_rows=growth_quantum_rows,
        )
        return self.finish(step.normalized, readings), state

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """Eval-only exact forward (no gradients: training stays on the reference)."""
        out, _ = self.prefill(tokens, growth_quantum_rows=max(16, tokens.shape[0] * self.memory_heads))
        return out
