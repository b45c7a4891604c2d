"""The whole ZONOS3-Mini LM on the B200 kernels, with the reference model's structure, checkpoint names and entry
points (``Zonos3ForCausalLM``, servers/sgl/src/zonos3_sgl/models/zonos3.py:1049-1360), and the captured decode step
the engine's graph runner replays (``DecodeGraph``, servers/sgl/src/zonos3_sgl/engine/graph.py).

A forward is:

    x      = zb_embed_norm(input_ids)                  multi-codebook embedding sum + emb_norm, one kernel
    h      = forward_layers_full(layers, x, ...)       the Full AttnRes schedule (attnres.py): a route before every
                                                        sublayer (OriginalGDN / Attention, then MoEFeedForward) and a
                                                        final route with out_norm, all routes over one bank
    logits = softcap(h @ multi_output^T)               [N, n_codebooks, audio_vocab]

``DecodeGraph`` captures one decode step of a fixed batch of streams as a single CUDA graph: embedding, the layer
stack, the head GEMM and ``sample_tts`` (soft cap fused into the sampler's load), then feeds the sampled codes back
as the next step's input ids, advances every stream's position and KV slot, and appends the codes to the
repetition-penalty window. ``step()`` is the end-to-end call: host ids and attention metadata in, host codes out.

Speaker / condition rows, hidden steering, accents and alignment probes of the reference model are not part of the
hot path and are not built.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib, ops
from .attention import Attention, SlotKVPool
from .attnres import FusedBlockAttnResContext, forward_layers_full
from .base import BaseOP, OPList, Weight
from .core import AttnMetadata, Batch, Req, forward_batch, get_global_ctx
from .gdn import OriginalGDN
from .moe import MoEFeedForward


class MultiEmbedding(BaseOP):
    """One table per audio codebook (audio_vocab rows) and one text table (text_vocab + 1 + extra rows);
    checkpoint names ``multi_embedder.embedders.{i}.weight`` (zonos3.py:186-255)."""

    def __init__(self, config):
        rows = [config.audio_vocab_size] * config.n_codebooks
        if config.text_vocab is not None:
            rows.append(config.text_vocab + 1 + int(config.text_extra_tokens))
        self.embedders = OPList([Weight((n, config.hidden_size)) for n in rows])

    def forward(self, codes: torch.Tensor, *, eps: float = 1e-5, norm_weight=None, normalize: bool = False,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Sum of the columns' rows (and, with ``normalize``, the embedding RMSNorm fused) for codes [N, C]."""
        tables = [e.weight for e in self.embedders.op_list]
        return ops.embed_norm(codes.to(torch.int32), tables, eps=eps, norm_weight=norm_weight, normalize=normalize,
                              out=out)


class FeedForward(BaseOP):
    """Dense SwiGLU FFN of layers before ``moe_start_from_layer``: first half times SiLU(second half)
    (w_in [2, I, D], w_out [D, I]; zonos3.py:393-420, lm.py:606-609). cuBLAS GEMMs: not on the MoE hot path."""

    def __init__(self, config):
        inter = config.intermediate_size
        self.w_in = Weight((2, inter, config.hidden_size))
        self.w_out = Weight((config.hidden_size, inter))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        inter = self.w_out.weight.shape[1]
        flat = F.linear(x, self.w_in.weight.reshape(2 * inter, -1))
        return F.linear(flat[:, :inter] * F.silu(flat[:, inter:]), self.w_out.weight)


class TransformerBlock(BaseOP):
    """attention_norm -> attention (gated DeltaNet or GQA) -> ffn_norm -> feed_forward (MoE or dense), wired by the
    Full AttnRes schedule (zonos3.py:885-960)."""

    def __init__(self, config, layer_id: int):
        D = config.hidden_size
        self.attention_norm = Weight((D,))
        self.attention = OriginalGDN(config, layer_id) if config.uses_gdn(layer_id) else Attention(config, layer_id)
        self.ffn_norm = Weight((D,))
        self.is_moe = config.is_moe(layer_id)
        self.feed_forward = MoEFeedForward(config, layer_id) if self.is_moe else FeedForward(config)


class Zonos3ForCausalLM(BaseOP):
    """Checkpoint names as the reference's (no "model." prefix): multi_embedder.*, layers.{i}.*, out_norm.weight,
    multi_output.weight, block_attnres_queries."""

    def __init__(self, config):
        self._config = config
        self.n_codebooks = config.n_codebooks
        self.audio_vocab = config.audio_vocab_size
        D, L = config.hidden_size, config.num_layers
        self.multi_embedder = MultiEmbedding(config)
        self.layers = OPList([TransformerBlock(config, i) for i in range(L)])
        self.block_attnres_queries = torch.empty(2 * L + 1, D)
        self.out_norm = Weight((D,))
        self.multi_output = Weight((self.n_codebooks * self.audio_vocab, D))
        self._attnres_states: dict = {}
        self._head = None  # multi_output.weight padded to a multiple of 8 rows (prepare())

    @property
    def config(self):
        return self._config

    def attention_layer_ids(self) -> list[int]:
        return [i for i, layer in enumerate(self.layers.op_list) if isinstance(layer.attention, Attention)]

    def gdn_layers(self) -> list[OriginalGDN]:
        return [layer.attention for layer in self.layers.op_list if isinstance(layer.attention, OriginalGDN)]

    def prepare(self) -> None:
        """Concatenated attention projections and the padded head (after the weights are loaded and on the device,
        before capture)."""
        for layer in self.layers.op_list:
            if isinstance(layer.attention, Attention):
                layer.attention.prepare()
        # the head's 10 x 4098 = 40980 outputs make a 81,960-byte row, which is not 16-byte aligned: cuBLAS then falls
        # back to a slow kernel (189 us instead of ~30 us at 256 rows); 4 zero rows make every logits row aligned
        w = self.multi_output.weight
        rows = (w.shape[0] + 7) // 8 * 8
        self._head = torch.zeros(rows, w.shape[1], device=w.device, dtype=w.dtype)
        self._head[: w.shape[0]].copy_(w)

    @property
    def head_rows(self) -> int:
        """Columns of the padded head output (the logits row stride)."""
        return (self.n_codebooks * self.audio_vocab + 7) // 8 * 8

    def allocate_caches(self, capacity: int, kv_slots: int, device) -> SlotKVPool:
        """Per-slot DeltaNet state pools of ``capacity`` streams and the KV pool of ``kv_slots`` token slots."""
        for gdn in self.gdn_layers():
            gdn.allocate_cache(capacity, device, torch.bfloat16)
        c = self._config
        return SlotKVPool(self.attention_layer_ids(), kv_slots, c.num_kv_heads, c.head_dim, device)

    # ------------------------------------------------------------------ forward pieces (zonos3.py:1159-1360)
    def embed(self, input_ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return self.multi_embedder.forward(input_ids, eps=self._config.rms_norm_eps, normalize=True, out=out)

    def _attnres_state(self, x: torch.Tensor, persistent: bool) -> FusedBlockAttnResContext:
        if not persistent:
            return FusedBlockAttnResContext(2 * len(self.layers.op_list), x, gradient_dtype=x.dtype)
        key = (x.shape[0], x.dtype, x.device)
        state = self._attnres_states.get(key)
        if state is None:
            state = FusedBlockAttnResContext(2 * len(self.layers.op_list), x, gradient_dtype=x.dtype)
            self._attnres_states[key] = state
        return state

    def forward_layers(self, x: torch.Tensor) -> torch.Tensor:
        batch = get_global_ctx().batch
        state = self._attnres_state(x, persistent=batch is not None and batch.is_decode)
        return forward_layers_full(self.layers.op_list, x, self.block_attnres_queries, self._config.rms_norm_eps,
                                   state, self.out_norm.weight)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        logits = F.linear(hidden, self.multi_output.weight).view(-1, self.n_codebooks, self.audio_vocab)
        cap = self._config.loss_softcap
        return cap * torch.tanh(logits / cap) if cap > 0 else logits

    def forward(self) -> torch.Tensor:
        return self.compute_logits(self.forward_layers(self.embed(get_global_ctx().batch.input_ids)))


# ------------------------------------------------------------------------------------------ captured decode step


@dataclass
class SamplingConfig:
    """Every stream's sampler settings (clamp_sampling, model/src/zonos3/tts/sampler.py:27-40); temperature <= 0 is
    greedy."""

    temperature: float = 0.8
    top_k: int = 50
    top_p: float = 0.9
    min_p: float = 0.0
    repetition_window: int = 32
    repetition_penalty: float = 1.2
    seed: int = 0


class DecodeGraph:
    """One decode step of ``batch_size`` streams as one CUDA graph (the engine's graph runner, engine/graph.py).

    Static device buffers hold the step's inputs: ``input_ids`` [B, C + 1] int32, the attention metadata
    (``positions``, ``out_loc``, ``cache_seqlens`` [B] int32 and ``page_table`` [B, max_len] int32), the DeltaNet
    state ``slots`` [B] int64. A replay runs the model and the sampler, then prepares the next step on the device:
    ``input_ids`` <- the sampled codes, every position and cache length + 1, ``out_loc`` <- the next slot of each
    stream's page table, the codes appended to the repetition window, the sampler's draw counter + 1. So replays
    alone run an autoregressive decode; ``step()`` instead loads host ids / metadata first (the server's path).
    """

    def __init__(self, model: Zonos3ForCausalLM, pool: SlotKVPool, batch_size: int, page_table: torch.Tensor,
                 slots: torch.Tensor | None = None, sampling: SamplingConfig | None = None, stop_id: int | None = None):
        c = model.config
        dev = page_table.device
        self.model, self.pool, self.bs = model, pool, batch_size
        self.C, self.V = c.n_codebooks, c.audio_vocab_size
        self.sampling = sampling or SamplingConfig()
        self.codebook_size = c.codebook_size
        self.audio_pad_id = c.audio_pad_id
        self.text_pad = c.text_vocab if c.text_vocab is not None else 0
        self.softcap = float(c.loss_softcap)
        i32 = dict(device=dev, dtype=torch.int32)
        B = batch_size
        if page_table.shape[0] != B or page_table.dtype != torch.int32:
            raise ValueError(f"page_table must be a [{B}, max_len] int32 tensor")
        self.page_table = page_table.contiguous()
        self.input_ids = torch.zeros(B, self.C + (c.text_vocab is not None), **i32)
        self.codes = torch.zeros(B, self.C + 1, **i32)
        self.positions = torch.zeros(B, **i32)
        self.out_loc = torch.zeros(B, **i32)
        self.cache_seqlens = torch.ones(B, **i32)
        self.slots = (torch.arange(B, device=dev, dtype=torch.int64) if slots is None else slots).contiguous()
        self.x = torch.empty(B, c.hidden_size, device=dev, dtype=torch.bfloat16)
        self.head_out = torch.empty(B, model.head_rows, device=dev, dtype=torch.bfloat16)  # row stride aligned
        self.logits = self.head_out[:, : self.C * self.V]  # [B, C * V] view; the sampler reads it in place
        W = max(int(self.sampling.repetition_window), 0)
        self.history = torch.full((B, self.C, max(W, 1)), -1, **i32)
        self.W = W
        self.ring = torch.zeros(1, device=dev, dtype=torch.int64)
        self.counter = torch.zeros(1, device=dev, dtype=torch.int64)
        self.temperatures = torch.full((B,), float(self.sampling.temperature), device=dev, dtype=torch.float32)
        self.stop_ids = torch.full((B,), c.codebook_size if stop_id is None else int(stop_id), **i32)
        self.penalties = torch.full((B,), float(self.sampling.repetition_penalty), device=dev, dtype=torch.float32)
        self.batch = Batch(reqs=[Req(i, 1, cached_len=1) for i in range(B)], is_decode=True, padded_size=B,
                           input_ids=self.input_ids,
                           attn_metadata=AttnMetadata(self.positions, self.out_loc, self.page_table, self.cache_seqlens))
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches_per_step = 0  # this library's kernels in the captured step
        for gdn in model.gdn_layers():
            gdn.enable_graph_decode(self.slots, OriginalGDN.static_tables(dev, [B]))
            gdn.set_static_mode(True)

    # ------------------------------------------------------------------ the captured body
    def _body(self) -> None:
        m, s = self.model, self.sampling
        x = m.embed(self.input_ids, out=self.x)
        h = m.forward_layers(x)
        torch.matmul(h, m._head.t(), out=self.head_out)
        ops.sample_tts(self.logits.unflatten(1, (self.C, self.V)), [s.temperature] * self.bs, [s.top_k], [s.top_p],
                       [s.min_p], codebook_size=self.codebook_size, audio_pad_id=self.audio_pad_id,
                       stop_token_ids=self.stop_ids,
                       repetition_token_ids=self.history if self.W and s.repetition_penalty > 1.0 else None,
                       repetition_penalties=self.penalties, text_vocab=self.text_pad, seed=s.seed,
                       offset_dev=self.counter, out=self.codes, device_temperatures=self.temperatures,
                       softcap=self.softcap)
        # the next step's inputs, on the device (one kernel)
        ops.decode_advance(self.codes, self.input_ids, self.positions, self.cache_seqlens, self.out_loc,
                           self.page_table, self.counter, history=self.history if self.W else None,
                           ring=self.ring if self.W else None)

    def _context(self):
        ctx = get_global_ctx()
        ctx.attn_backend = self.pool
        return forward_batch(self.batch)

    def capture(self, warmup: int = 1) -> None:
        """Runs the body eagerly ``warmup`` times (library handles, workspaces), then captures it. The warm-up runs
        advance the streams' states: capture before loading the streams (the engine captures at start-up)."""
        self.model.prepare()
        stream = torch.cuda.Stream(self.page_table.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream), self._context():
            for _ in range(warmup):
                self._body()
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            before = _lib.launch_count()
            with torch.cuda.graph(self.graph, stream=stream):
                self._body()
            self.launches_per_step = _lib.launch_count() - before
        torch.cuda.current_stream().wait_stream(stream)
        self.reset()

    def reset(self) -> None:
        """Clears the repetition window and the draw counter (a fresh set of streams)."""
        self.history.fill_(-1)
        self.ring.zero_()
        self.counter.zero_()

    def load(self, input_ids=None, positions=None, cache_seqlens=None, out_loc=None) -> None:
        """Copies new step inputs into the static buffers (host tensors should be pinned; copies are asynchronous on
        the current stream)."""
        for dst, src in ((self.input_ids, input_ids), (self.positions, positions), (self.cache_seqlens, cache_seqlens),
                         (self.out_loc, out_loc)):
            if src is not None:
                dst.copy_(src, non_blocking=True)

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("DecodeGraph.capture() first")
        get_global_ctx().attn_backend = self.pool
        self.graph.replay()
        return self.codes

    def step(self, host_ids: torch.Tensor, host_codes: torch.Tensor, positions=None, cache_seqlens=None,
             out_loc=None) -> torch.Tensor:
        """End to end: host ids [B, C + 1] (pinned) and optional host metadata in, replay, sampled codes copied
        into the pinned host tensor ``host_codes`` [B, C + 1] (asynchronous; synchronise before reading)."""
        self.load(host_ids, positions, cache_seqlens, out_loc)
        self.replay()
        host_codes.copy_(self.codes, non_blocking=True)
        return host_codes
