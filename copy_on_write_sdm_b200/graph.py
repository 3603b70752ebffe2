"""CUDA-graph replay of whole-model decode.

``LanguageModel.decode`` (reference model.py:436-466 -> inference.py:601-669)
issues a few hundred small kernels per token -- layer norms, projections,
product-key top-k, the fused packed SDM step of every "B" layer, K/V-cache
attention, MLPs and the vocabulary head -- plus host checks.  At serving batch
sizes the host, not the GPU, sets the step time.  ``GraphedDecode`` captures
one decode token of the whole stack into a CUDA graph and replays it:

* inputs are two static device buffers (token ids ``[B,1]`` and positions
  ``[B]``); the logits come back in a static ``[B,1,vocab]`` buffer that the
  next step overwrites;
* attention reads the whole fixed-capacity K/V cache under a mask built on the
  device from the positions, so one graph serves every position (the eager
  path slices the cache to ``position+1`` instead; softmax weights of masked
  slots are exactly zero, so only the summation order differs);
* the packed SDM steps are the same ``cow_decode_step`` launches as the eager
  path (pool descriptors are baked into the graph);
* the host does the reference's per-step bookkeeping before each replay: the
  capacity checks and the capacity proof (``prepare_step_capacity``,
  allocator.py:746-774) of every pool.  When any pool or cache tensor was
  replaced (growth, trim, admission, compaction) the step runs eagerly and the
  graph is captured again.

Semantics per step equal ``LanguageModel.decode`` on the same state; the
state object stays usable by the eager API between replays.
"""

from __future__ import annotations

import torch

from .allocator import new_decode_scratch, packed_sdm_cow_step
from .inference import FaithfulSDMDecodeState, _step_kwargs


def _attend_full(attention, tokens: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 pos: torch.Tensor) -> torch.Tensor:
    """One-token attention over the whole cache; slots after each request's position are masked."""
    q, k, v = attention.project_qkv(tokens)
    rows = torch.arange(tokens.shape[0], device=tokens.device)
    key_cache[rows, :, pos] = k[:, :, 0]
    value_cache[rows, :, pos] = v[:, :, 0]
    capacity = key_cache.shape[2]
    hidden = torch.arange(capacity, device=tokens.device)[None, :] > pos[:, None]
    mask = torch.zeros(tokens.shape[0], 1, 1, capacity, device=tokens.device, dtype=q.dtype)
    mask.masked_fill_(hidden[:, None, None, :], float("-inf"))
    return attention._merge(attention._sdpa(q, key_cache, value_cache, causal=False, mask=mask))


class GraphedDecode:
    """Decode ``state`` through ``model`` by CUDA-graph replay (see the module docstring)."""

    def __init__(self, model, state: FaithfulSDMDecodeState) -> None:
        if model.training:
            raise ValueError("graphed decode requires model.eval()")
        if state.layout != model.stack.layout:
            raise ValueError("decode state layout does not match the model")
        if state.device.type != "cuda":
            raise ValueError("graphed decode runs on a CUDA device")
        self.model, self.state = model, state
        self.device = state.device
        self._graph: torch.cuda.CUDAGraph | None = None
        self._key = None
        self._alloc(state.batch)
        self.replays = 0
        self.captures = 0
        self._active_ok = None  # key of the active-flags tensor last found all true

    def _alloc(self, batch: int) -> None:
        self.batch = batch
        self.ids = torch.zeros(batch, 1, dtype=torch.int64, device=self.device)
        self.pos = torch.zeros(batch, dtype=torch.int64, device=self.device)
        self.logits = None
        # Look-back scratch owned by this decoder: a captured graph keeps its
        # address, so it must live exactly as long as the graphs that use it
        # (a batch change replaces it and forces a new capture).
        banks = max((st.banks for st in self.state.sdm_states), default=0)
        self.scratch = new_decode_scratch(self.device, max(banks, 1), 1)

    def _tensor_key(self):
        """What the captured graph depends on: the batch, each pool object and its
        tensor-replacement counter (slab, map, stack, counters; capacity follows the
        slab view) and the K/V cache tensors.  Objects are keyed by identity and kept
        referenced with the graph (``_key_refs``), so an id in a held key cannot be
        reused by another object."""
        s = self.state
        objs = (*s.sdm_states, *s.dense_keys, *s.dense_values)
        return (s.batch, tuple(id(o) for o in objs),
                tuple(st.__dict__.get("_tensor_version", 0) for st in s.sdm_states)), objs

    def _body(self) -> torch.Tensor:
        """One token through the stack, reading ``self.ids`` / ``self.pos``."""
        model, state, stack = self.model, self.state, self.model.stack
        tokens = model._embed(self.ids, self.pos[:, None])
        a_i = b_i = 0
        for i, kind in enumerate(stack.layout):
            if kind == "A":
                block = stack.attention_layers[str(i)]
                kc, vc = state.dense_keys[a_i], state.dense_values[a_i]
                if block._fused_decode_ok(tokens, kc, vc):
                    tokens = block.decode_residual(tokens, kc, vc, self.pos)
                else:
                    tokens = tokens + _attend_full(block.attention, tokens, kc, vc, self.pos)
                    tokens = tokens + block.mlp(tokens)
                a_i += 1
                continue
            module = stack.sdm_layers[str(i)]
            step = module.controller(tokens)
            reading, _ = packed_sdm_cow_step(state.sdm_states[b_i], **_step_kwargs(step), validate_routes=False,
                                             collect_diagnostics=False, scratch=self.scratch)
            tokens = module.finish_residual(tokens, step.normalized, reading[:, None], stack.sdm_mlps[str(i)])
            b_i += 1
        return model.output(model.final_norm(tokens))

    def _check(self, input_ids: torch.Tensor) -> None:
        state, model = self.state, self.model
        if input_ids.shape != (state.batch, 1):
            raise ValueError(f"decode input_ids must be [{state.batch},1]")
        if state.position >= model.maximum_sequence_length:
            raise ValueError("sequence exceeds maximum_sequence_length")
        if state.position >= state.capacity:
            raise ValueError("decode state has reached its fixed capacity")
        # The reference reads the active flags every token (a host synchronisation);
        # they change only through assignments or in-place tensor ops, so one
        # passing check holds until the tensor object or its version changes.
        act = state.active_sequences
        ok = self._active_ok
        if ok is None or ok[0] is not act or ok[1] != act._version:
            if not bool(act.all()):
                raise ValueError("released requests must be removed before further decode")
            self._active_ok = (act, act._version)  # holds the tensor, so its identity cannot be reused
        for st, module in zip(state.sdm_states, (model.stack.sdm_layers[str(i)] for i in state.sdm_layer_positions)):
            if st.banks != state.batch * module.memory_heads:
                raise ValueError("packed SDM banks do not match batch and memory heads")
            if st.growth_quantum_rows:
                st.prepare_step_capacity(st.banks * module.writes)

    @torch.no_grad()
    def step(self, input_ids: torch.Tensor) -> torch.Tensor:
        """One decode token for every request; returns the static logits buffer ``[B,1,vocab]``."""
        state = self.state
        if any(not st.growth_quantum_rows and not st.capacity_is_proven for st in state.sdm_states):
            # A fixed pool without a decode proof (e.g. after admission) takes the
            # reference's checked path, which reads the status word every step.
            return self.model.decode(input_ids, state)
        self._check(input_ids)
        if state.batch != self.batch:
            self._alloc(state.batch)
        self.ids.copy_(input_ids, non_blocking=True)
        if state.positions is None:
            self.pos.fill_(state.position)
        else:
            self.pos.copy_(state.positions)
        key, objs = self._tensor_key()
        if key != self._key or self._graph is None:
            # Eager step (it is this token's real step), then capture for the next ones.
            self._graph = None
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                logits = self._body()
            torch.cuda.current_stream(self.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self.logits = self._body()
            self._graph, self._key, self._key_refs = graph, key, objs
            self.captures += 1
            self.logits.copy_(logits)
        else:
            self._graph.replay()
            self.replays += 1
        if state.positions is None:
            state.position += 1
        else:
            state.positions = state.positions + 1
            state.position += 1
        return self.logits
