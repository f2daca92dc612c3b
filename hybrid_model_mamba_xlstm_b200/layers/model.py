"""Hybrid Mamba / xLSTM language model (prefill forward) on the hxm kernels.

Mirrors HybridConfig (hybrid_xmamba/models/configuration_hybrid.py:11-111)
and HybridLanguageModel.forward (hybrid_xmamba/models/hybrid_lm.py:88-209):
embedding -> HybridBlocks cycling ``layer_pattern`` -> final RMSNorm ->
lm_head.  State-dict keys match the reference.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.nn as nn

from .blocks import HybridBlock, RMSNorm


@dataclass
class HybridConfig:
    """Fields and defaults of the reference HybridConfig (:47-111), plus
    ``slstm_recurrent`` (block-diagonal recurrent weights in sLSTM layers)
    and ``residual_init_scale`` (scale residual-out projections by
    1/sqrt(2 * num_layers) at init)."""
    vocab_size: int = 50257
    dim: int = 768
    num_layers: int = 12
    layer_pattern: List[str] = field(default_factory=lambda: ["mamba", "mamba", "mlstm"])
    state_size: int = 16
    conv_size: int = 4
    expand_factor: int = 2
    dt_rank: Optional[int] = None
    use_fast_path: bool = True
    head_dim: int = 64
    num_heads: Optional[int] = None
    use_tfla: bool = True
    proj_factor: int = 2
    slstm_hidden_dim: Optional[int] = None
    slstm_num_heads: int = 4
    use_exponential_gate: bool = True
    norm_type: str = "rms"
    use_mlp: bool = True
    mlp_ratio: float = 4.0
    max_position_embeddings: int = 2048
    dropout: float = 0.1
    initializer_range: float = 0.02
    use_cache: bool = True
    tie_word_embeddings: bool = False
    slstm_recurrent: bool = False
    residual_init_scale: bool = False

    def __post_init__(self):
        if self.num_heads is None:
            self.num_heads = max(1, self.dim // self.head_dim)
        if self.dt_rank is None:
            self.dt_rank = max(1, self.dim // 16)
        if self.slstm_hidden_dim is None:
            self.slstm_hidden_dim = self.dim
        for t in self.layer_pattern:
            if t not in ("mamba", "mlstm", "slstm"):
                raise ValueError(f"Invalid layer type '{t}'")


def hybrid_350m_config(**over) -> HybridConfig:
    """d_model 1024, 24 layers of [Mamba, Mamba, mLSTM, sLSTM]; Mamba expand 2,
    d_state 16, conv 4; mLSTM 4 heads of 512; sLSTM 4 heads with block-diagonal
    recurrent weights; vocab 50304; residual projections scaled 1/sqrt(48)."""
    kw = dict(vocab_size=50304, dim=1024, num_layers=24, layer_pattern=["mamba", "mamba", "mlstm", "slstm"],
              state_size=16, conv_size=4, expand_factor=2, head_dim=512, num_heads=4, slstm_num_heads=4,
              dropout=0.0, slstm_recurrent=True, residual_init_scale=True)
    kw.update(over)
    return HybridConfig(**kw)


class HybridLanguageModel(nn.Module):
    def __init__(self, config: HybridConfig):
        super().__init__()
        self.config = c = config
        self.embeddings = nn.Module()
        self.embeddings.token_embedding = nn.Embedding(c.vocab_size, c.dim)
        self.layers = nn.ModuleList([
            HybridBlock(c.dim, layer_type=c.layer_pattern[i % len(c.layer_pattern)], norm_type=c.norm_type,
                        use_mlp=c.use_mlp, mlp_ratio=c.mlp_ratio, state_size=c.state_size, conv_size=c.conv_size,
                        expand_factor=c.expand_factor, dt_rank=c.dt_rank, use_fast_path=c.use_fast_path,
                        head_dim=c.head_dim, num_heads=c.num_heads, use_tfla=c.use_tfla, proj_factor=c.proj_factor,
                        slstm_hidden_dim=c.slstm_hidden_dim, slstm_num_heads=c.slstm_num_heads,
                        use_exponential_gate=c.use_exponential_gate, slstm_recurrent=c.slstm_recurrent)
            for i in range(c.num_layers)])
        self.final_norm = RMSNorm(c.dim) if c.norm_type.lower() == "rms" else nn.LayerNorm(c.dim)
        self.lm_head = nn.Linear(c.dim, c.vocab_size, bias=False)
        if c.tie_word_embeddings:
            self.lm_head.weight = self.embeddings.token_embedding.weight
        self.apply(self._init_weights)
        if c.residual_init_scale:
            s = 1.0 / math.sqrt(2 * c.num_layers)
            with torch.no_grad():
                for blk in self.layers:
                    blk.mixer.out_proj.weight.mul_(s)
                    if blk.mlp is not None:
                        blk.mlp[2].weight.mul_(s)
        if c.slstm_recurrent:
            with torch.no_grad():
                for blk in self.layers:
                    rw = getattr(blk.mixer, "recurrent_weight", None)
                    if rw is not None:
                        rw.normal_(0.0, 1.0 / math.sqrt(blk.mixer.head_dim))

    def _init_weights(self, module):
        """N(0, initializer_range) weights, zero biases (hybrid_lm.py:136-143)."""
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=self.config.initializer_range)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=self.config.initializer_range)

    def init_caches(self):
        """Empty per-layer recurrent caches (zero states) for :meth:`forward` / :meth:`generate`."""
        return [dict() for _ in self.layers]

    def forward(self, input_ids, return_hidden=False, caches=None):
        """Logits (B, L, vocab).  With ``caches`` (from :meth:`init_caches`) every
        layer starts from and updates its recurrent state (Mamba conv inputs and
        scan state, mLSTM (C, n, m), sLSTM (h, c)), so a sequence can be fed in
        pieces — the prefill / decode split of :meth:`generate`."""
        h = self.embeddings.token_embedding(input_ids)
        pending = None  # each block's last residual add is fused into the next RMSNorm
        for i, layer in enumerate(self.layers):
            h, pending = layer.forward_pending(h, pending, cache=None if caches is None else caches[i])
        if pending is None:
            h = self.final_norm(h)
        elif isinstance(self.final_norm, RMSNorm):
            h, _ = self.final_norm(pending, residual=h)
        else:
            h = self.final_norm(h + pending)
        if return_hidden:
            return h
        return self.lm_head(h)

    @staticmethod
    def _piece_bounds(L, pieces):
        """[(start, end)] of the wavefront's sequence pieces: ``pieces`` equal
        pieces of whole 128-step chunks, or explicit piece lengths (a sequence
        of ints; the last piece takes whatever of L is left)."""
        if isinstance(pieces, int):
            if pieces <= 1 or L < 2 * pieces:
                return [(0, L)]
            step = -(-L // pieces)
            step = -(-step // 128) * 128  # whole 128-step chunks per piece
            return [(a, min(a + step, L)) for a in range(0, L, step)]
        bounds, a = [], 0
        for n in pieces:
            if a >= L:
                break
            if n <= 0:
                raise ValueError(f"prefill: piece lengths must be positive, got {list(pieces)}")
            bounds.append((a, min(a + int(n), L)))
            a += int(n)
        if a < L:
            bounds.append((a, L))
        return bounds

    @torch.no_grad()
    def prefill(self, input_ids, pieces=4, caches=None, return_hidden=False):
        """Logits of :meth:`forward`, scheduled as a wavefront over layers and
        sequence pieces: the sequence is cut into ``pieces`` consecutive pieces,
        layer i runs on its own CUDA stream and takes piece k once layer i-1 has
        finished piece k (its own piece k-1 is done by stream order, the
        recurrent states carried in ``caches``).  The recurrences are exact
        across pieces (the same continuation as :meth:`forward` with caches), so
        the result is the whole-sequence forward; what changes is that layers
        working on different pieces run concurrently — the sLSTM recurrence
        occupies 8 SMs per head for thousands of sequential steps, and the other
        layers' kernels fill the rest of the GPU meanwhile.  On CPU, or with one
        piece, this is :meth:`forward`.  ``pieces`` may also list the piece
        lengths: a short first piece shortens the pipeline fill (the time until
        the last layer sees its first piece), which dominates at batch 1."""
        L = input_ids.shape[1]
        if caches is None:
            caches = self.init_caches()
        bounds = self._piece_bounds(L, pieces)
        if not input_ids.is_cuda or len(bounds) <= 1:
            return self.forward(input_ids, return_hidden=return_hidden, caches=caches)
        dev = input_ids.device
        main = torch.cuda.current_stream(dev)
        nl = len(self.layers)
        streams = [torch.cuda.Stream(dev) for _ in range(nl + 1)]
        start = torch.cuda.Event()
        start.record(main)
        for s in streams:
            s.wait_event(start)
        outs = [None] * len(bounds)
        for k, (a, b) in enumerate(bounds):
            ev = None
            with torch.cuda.stream(streams[0]):
                h = self.embeddings.token_embedding(input_ids[:, a:b])
            pending = None
            for i, layer in enumerate(self.layers):
                st = streams[i]
                with torch.cuda.stream(st):
                    if ev is not None:
                        st.wait_event(ev)
                    h, pending = layer.forward_pending(h, pending, cache=caches[i])
                    ev = torch.cuda.Event()
                    ev.record(st)
                # the activations move on to the next layer's stream: the allocator
                # must not hand their memory out again before that stream used them
                nxt = streams[i + 1]
                h.record_stream(nxt)
                if pending is not None:
                    pending.record_stream(nxt)
            st = streams[nl]
            with torch.cuda.stream(st):
                st.wait_event(ev)
                if pending is None:
                    y = self.final_norm(h)
                elif isinstance(self.final_norm, RMSNorm):
                    y, _ = self.final_norm(pending, residual=h)
                else:
                    y = self.final_norm(h + pending)
                outs[k] = y if return_hidden else self.lm_head(y)
                outs[k].record_stream(main)
        for s in streams:
            main.wait_stream(s)
        return torch.cat(outs, dim=1)

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens=100, temperature=1.0, top_k=None, top_p=None, cuda_graph=True):
        """Autoregressive sampling with the reference's interface and sampling rule
        (hybrid_xmamba/models/hybrid_lm.py:211-267), but one prefill over the
        prompt and then one single-token step per new token on the carried
        recurrent states, instead of re-running the whole prefix per token.
        With ``cuda_graph`` the single-token step (a few hundred small kernel
        launches) is captured once and replayed (:class:`GraphDecoder`)."""
        self.eval()
        if cuda_graph and input_ids.is_cuda and max_new_tokens > 1:
            dec = GraphDecoder(self, input_ids.shape[0], input_ids.device)
            logits = dec.prefill(input_ids)[:, -1, :]
            step = dec.step
        else:
            caches = self.init_caches()
            logits = self.forward(input_ids, caches=caches)[:, -1, :]
            step = lambda t: self.forward(t, caches=caches)
        out = [input_ids]
        for i in range(max_new_tokens):
            next_token_logits = logits.float() / temperature
            if top_k is not None:
                kth = torch.topk(next_token_logits, top_k)[0][..., -1, None]
                next_token_logits = next_token_logits.masked_fill(next_token_logits < kth, float("-inf"))
            if top_p is not None:
                sorted_logits, sorted_idx = torch.sort(next_token_logits, descending=True)
                cum = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
                drop = cum > top_p
                drop[..., 1:] = drop[..., :-1].clone()
                drop[..., 0] = False
                next_token_logits = next_token_logits.masked_fill(drop.scatter(1, sorted_idx, drop), float("-inf"))
            nxt = torch.multinomial(torch.softmax(next_token_logits, dim=-1), num_samples=1)
            out.append(nxt)
            if i + 1 < max_new_tokens:
                logits = step(nxt)[:, -1, :]
        return torch.cat(out, dim=1)


class PrefillGraph:
    """:meth:`HybridLanguageModel.prefill` of one (batch, seqlen) shape captured
    once into a CUDA graph and replayed: the wavefront's thousands of kernel
    launches across the per-layer streams cost no host time on replay, and the
    graph keeps the event dependencies between layers and pieces, so the GPU
    runs layers of different pieces concurrently.  ``__call__`` copies the
    token ids into the graph's input buffer and returns the graph's logits
    buffer (overwritten by the next call); :meth:`states` returns copies of
    the recurrent states after the prompt, to continue the sequence with
    :meth:`HybridLanguageModel.forward` (the graph's own state buffers must
    stay in place for the next replay)."""

    def __init__(self, model, batch, seqlen, pieces=4, device="cuda"):
        self.model, self.pieces = model, pieces
        dev = torch.device(device)
        self.ids = torch.zeros(batch, seqlen, dtype=torch.long, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            model.prefill(self.ids, pieces=pieces)  # warm-up: parameter caches, workspaces, kernel setup
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.caches = model.init_caches()
            self.logits = model.prefill(self.ids, pieces=pieces, caches=self.caches)

    def __call__(self, input_ids):
        self.ids.copy_(input_ids)
        self.graph.replay()
        return self.logits

    def states(self):
        """Per-layer caches (copies) holding the states after the last replay."""
        return [{k: v.clone() for k, v in c.items()} for c in self.caches]


class GraphDecoder:
    """Single-token decode of a :class:`HybridLanguageModel` replayed from one CUDA graph.

    The recurrent states live in static buffers; the captured step reads them,
    runs every layer on one token (its hxm kernels and cuBLAS GEMMs) and copies
    the new states back into the same buffers, so each replay advances the
    sequence by one token with no per-kernel launch overhead on the host."""

    def __init__(self, model, batch, device):
        self.model, self.batch, self.device = model, batch, torch.device(device)
        self.graph = None
        self.states = None
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=self.device)

    @torch.no_grad()
    def prefill(self, input_ids):
        caches = self.model.init_caches()
        logits = self.model(input_ids, caches=caches)
        self.states = [{k: v.clone() for k, v in c.items()} for c in caches]
        self.graph = None
        return logits

    def _run(self):
        caches = [dict(c) for c in self.states]
        logits = self.model(self.ids, caches=caches)
        for dst, src in zip(self.states, caches):
            for k, v in src.items():
                dst[k].copy_(v)
        return logits

    @torch.no_grad()
    def _capture(self):
        saved = [{k: v.clone() for k, v in c.items()} for c in self.states]
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(2):  # warm-up (lazy library setup, workspace sizes) on scratch states
                self._run()
        torch.cuda.current_stream(self.device).wait_stream(side)
        for dst, src in zip(self.states, saved):
            for k, v in src.items():
                dst[k].copy_(v)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._run()

    @torch.no_grad()
    def step(self, token_ids):
        """Logits (batch, 1, vocab) of the next position after feeding `token_ids` (batch, 1)."""
        if self.states is None:
            raise RuntimeError("GraphDecoder.step before prefill")
        self.ids.copy_(token_ids)
        if self.graph is None:
            self._capture()
        self.graph.replay()
        return self.logits
