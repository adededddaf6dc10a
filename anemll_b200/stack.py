"""The 24-layer hybrid decoder stack on one GPU (or one shard of sequences per rank).

Embedding -> 24 layers -> final RMSNorm -> LM head -> in-model argmax (greedy next token).  Layer i
is a full-attention layer iff (i + 1) % 4 == 0 (18 gated-DeltaNet layers, 6 attention layers), each
followed by a SwiGLU MLP, both pre-normed (RMSNorm) with residuals.

* Gated-DeltaNet layers: :class:`anemll_b200.gdn.GatedDeltaNet` (the library's prologue, chunked
  prefill / recurrent decode and gated RMSNorm kernels between torch projections).
* Attention layers: the Qwen3.5 gated full attention in the reference's shape (H_q 16, H_kv 2,
  head_dim 256): one fused q/k/v projection (q_proj also yields the sigmoid gate), then
  :func:`anemll_b200.attention.kv_attention_qkv`, which applies the per-head RMSNorm of q and k
  (``QwenHeadNorm``, ``anemll/models/qwen_model.py:143-184``) and the rotary embedding
  (``apply_rotary_pos_emb``, 186-261) inside the attention call, writes the new cache rows and applies
  the gate in its epilogue; then o_proj.
* Projections and the LM head: torch's GEMM (``F.linear``); norms and the SwiGLU: the one-pass
  kernels of ``stack_ops.cu``.

Caches and states are per sequence: KV caches ``[B, H_kv, ctx, hd]`` per attention layer, conv and
recurrent states per GDN layer.  Weights are random N(0, 0.02) (no checkpoints offline).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, attention, gdn

__all__ = ["StackConfig", "HybridStack", "GreedyDecoder", "nccl_id_gather", "shard", "rms_norm", "silu_mul",
           "rope_tables"]


class StackConfig:
    def __init__(self, n_layers=24, hidden=2048, ffn=6144, vocab=151936, ctx=4096, H_qk=16, H_v=32, d_k=128, d_v=128,
                 H_q=16, H_kv=2, head_dim=256, rope_theta=1e7, eps=1e-6):
        self.n_layers, self.hidden, self.ffn, self.vocab, self.ctx = n_layers, hidden, ffn, vocab, ctx
        self.H_qk, self.H_v, self.d_k, self.d_v = H_qk, H_v, d_k, d_v
        self.H_q, self.H_kv, self.head_dim = H_q, H_kv, head_dim
        self.rope_theta, self.eps = rope_theta, eps

    def is_attention(self, i):
        return (i + 1) % 4 == 0


def rms_norm(x, w, eps, residual=None):
    """RMSNorm over the last dim (fp32 arithmetic, one rounding): ``anemll_rmsnorm``.  With
    ``residual``: ``s = x + residual`` (rounded) first; returns ``(s, norm(s))``."""
    _need_cuda(x)
    d = x.shape[-1]
    x = x.contiguous()
    out = torch.empty_like(x)
    rows = x.numel() // d
    lib = _lib.load()
    if residual is None:
        rc = lib.anemll_rmsnorm(_lib.ptr(x), None, None, _lib.ptr(w), _lib.ptr(out), _lib.dtype_code(x.dtype), rows, d,
                                float(eps), _lib.stream_ptr(x.device))
        _lib.check(rc, "anemll_rmsnorm")
        return out
    residual = residual.contiguous()
    s = torch.empty_like(x)
    rc = lib.anemll_rmsnorm(_lib.ptr(x), _lib.ptr(residual), _lib.ptr(s), _lib.ptr(w), _lib.ptr(out),
                            _lib.dtype_code(x.dtype), rows, d, float(eps), _lib.stream_ptr(x.device))
    _lib.check(rc, "anemll_rmsnorm")
    return s, out


def silu_mul(gate_up):
    """SwiGLU of a ``[..., 2 ffn]`` gate|up projection: ``silu(gate) * up`` (``anemll_silu_mul``)."""
    _need_cuda(gate_up)
    gate_up = gate_up.contiguous()
    ffn = gate_up.shape[-1] // 2
    out = torch.empty(*gate_up.shape[:-1], ffn, dtype=gate_up.dtype, device=gate_up.device)
    rc = _lib.load().anemll_silu_mul(_lib.ptr(gate_up), _lib.ptr(out), _lib.dtype_code(gate_up.dtype),
                                     gate_up.numel() // (2 * ffn), ffn, _lib.stream_ptr(gate_up.device))
    _lib.check(rc, "anemll_silu_mul")
    return out


def _need_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("anemll_b200 ops take CUDA tensors (no CPU path)")


def rope_tables(dim, n_pos, theta, device):
    """cos/sin [n_pos, dim] (fp32, computed in fp64) of the rotary embedding, both halves equal."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64, device=device) / dim))
    t = torch.arange(n_pos, dtype=torch.float64, device=device)
    f = torch.outer(t, inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().float(), emb.sin().float()


class GatedAttention(nn.Module):
    """Gated full attention.  q_proj, k_proj and v_proj are views of one fused [q|k|v] weight, so the
    projections are one GEMM whose output the attention call reads in place (head norm and RoPE
    fused in), or ``anemll_qk_norm_rope`` for shapes the fused call does not take."""

    def __init__(self, cfg: StackConfig, device, dtype):
        super().__init__()
        fk = dict(device=device, dtype=dtype)
        self.cfg = cfg
        Hq, Hkv, hd = cfg.H_q, cfg.H_kv, cfg.head_dim
        self.n_q, self.n_kv = Hq * hd * 2, Hkv * hd  # q_proj rows per head: [query | gate]
        self.w_qkv = torch.empty(self.n_q + 2 * self.n_kv, cfg.hidden, **fk)
        self.q_proj = nn.Linear(cfg.hidden, self.n_q, bias=False, device="meta")
        self.k_proj = nn.Linear(cfg.hidden, self.n_kv, bias=False, device="meta")
        self.v_proj = nn.Linear(cfg.hidden, self.n_kv, bias=False, device="meta")
        self.q_proj.weight = nn.Parameter(self.w_qkv[:self.n_q])
        self.k_proj.weight = nn.Parameter(self.w_qkv[self.n_q:self.n_q + self.n_kv])
        self.v_proj.weight = nn.Parameter(self.w_qkv[self.n_q + self.n_kv:])
        self.o_proj = nn.Linear(Hq * hd, cfg.hidden, bias=False, **fk)
        self.q_norm = nn.Parameter(torch.ones(hd, device=device))
        self.k_norm = nn.Parameter(torch.ones(hd, device=device))

    def project(self, x, cos, sin, pos):
        """q [B, H_q, T, hd], k/v [B, H_kv, T, hd] (normed, rotated), gate [B, T, H_q*hd], from one fused
        q/k/v GEMM and ``anemll_qk_norm_rope`` (the unfused prologue)."""
        return self._prologue(F.linear(x, self.w_qkv), cos, sin, pos)

    def _prologue(self, qkv, cos, sin, pos):
        B, T, ld = qkv.shape
        c = self.cfg
        q = torch.empty(B, c.H_q, T, c.head_dim, dtype=qkv.dtype, device=qkv.device)
        k = torch.empty(B, c.H_kv, T, c.head_dim, dtype=qkv.dtype, device=qkv.device)
        v = torch.empty_like(k)
        gate = torch.empty(B, T, c.H_q * c.head_dim, dtype=qkv.dtype, device=qkv.device)
        base = qkv.data_ptr()
        es = qkv.element_size()
        rc = _lib.load().anemll_qk_norm_rope(
            base, ld, base + self.n_q * es, ld, base + (self.n_q + self.n_kv) * es, ld, _lib.ptr(self.q_norm),
            _lib.ptr(self.k_norm), _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(gate),
            _lib.dtype_code(qkv.dtype), B, T, c.H_q, c.H_kv, c.head_dim, int(pos), float(c.eps),
            _lib.stream_ptr(qkv.device))
        _lib.check(rc, "anemll_qk_norm_rope")
        return q, k, v, gate

    def forward(self, x, k_cache, v_cache, pos, cos, sin, fused=True):
        """``cos``/``sin``: the whole [ctx, hd] tables; this call's rows start at ``pos``.  ``fused``: the
        head norm and RoPE run inside the attention call (``anemll_kv_attention_qkv``) where it takes
        the shape, else through the separate prologue kernel."""
        c = self.cfg
        qkv = F.linear(x, self.w_qkv)  # [B, T, n_q + 2 n_kv]
        o = None
        if fused:
            o = attention.kv_attention_qkv(qkv, self.q_norm, self.k_norm, cos, sin, c.eps, k_cache, v_cache, pos,
                                           c.H_q, c.H_kv, c.head_dim)
        if o is None:
            q, k, v, gate = self._prologue(qkv, cos, sin, pos)
            o = attention.kv_attention(q, k_cache, v_cache, pos, k_new=k, v_new=v, gate=gate)
        return F.linear(o, self.o_proj.weight)


class HybridStack(nn.Module):
    def __init__(self, cfg: StackConfig = None, device="cuda", dtype=torch.bfloat16):
        super().__init__()
        cfg = cfg or StackConfig()
        self.cfg, self.dtype = cfg, dtype
        fk = dict(device=device, dtype=dtype)
        self.embed = nn.Embedding(cfg.vocab, cfg.hidden, **fk)
        self.mixers = nn.ModuleList()
        self.gate_up = nn.ModuleList()
        self.down = nn.ModuleList()
        self.norm1 = nn.ParameterList()
        self.norm2 = nn.ParameterList()
        for i in range(cfg.n_layers):
            if cfg.is_attention(i):
                self.mixers.append(GatedAttention(cfg, device, dtype))
            else:
                self.mixers.append(gdn.GatedDeltaNet(cfg.hidden, cfg.H_qk, cfg.H_v, cfg.d_k, cfg.d_v, device=device,
                                                     dtype=dtype))
            self.gate_up.append(nn.Linear(cfg.hidden, 2 * cfg.ffn, bias=False, **fk))
            self.down.append(nn.Linear(cfg.ffn, cfg.hidden, bias=False, **fk))
            self.norm1.append(nn.Parameter(torch.ones(cfg.hidden, device=device)))
            self.norm2.append(nn.Parameter(torch.ones(cfg.hidden, device=device)))
        self.norm = nn.Parameter(torch.ones(cfg.hidden, device=device))
        self.lm_head = nn.Linear(cfg.hidden, cfg.vocab, bias=False, **fk)
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.ctx, cfg.rope_theta, device)

    @torch.no_grad()
    def init_weights(self, seed=4):
        """Random-init weights ~N(0, 0.02) (norm gains 1; GDN conv ~N(0, 0.1), A_log ~U(0, log 16))."""
        g = torch.Generator(device=self.lm_head.weight.device)
        g.manual_seed(seed)
        for name, p in self.named_parameters():
            if "norm" in name and p.dim() == 1:
                p.fill_(1.0)
            elif name.endswith("conv_weight"):
                p.copy_(torch.randn(p.shape, generator=g, device=p.device) * 0.1)
            elif name.endswith("A_log"):
                p.copy_(torch.rand(p.shape, generator=g, device=p.device) * math.log(16.0))
            elif name.endswith("dt_bias"):
                p.zero_()
            else:
                p.copy_((torch.randn(p.shape, generator=g, device=p.device, dtype=torch.float32) * 0.02).to(p.dtype))
        return self

    def new_state(self, B):
        """Per-sequence caches and states for B sequences (zeroed)."""
        c, dev = self.cfg, self.lm_head.weight.device
        st = []
        for m in self.mixers:
            if isinstance(m, GatedAttention):
                k = torch.zeros(B, c.H_kv, c.ctx, c.head_dim, device=dev, dtype=self.dtype)
                st.append((k, torch.zeros_like(k)))
            else:
                st.append(m.new_states(B))
        return st

    def mixer(self, i, h, state, pos):
        """Layer i's attention or gated-DeltaNet block on its normed input h [B, T, hidden]."""
        m = self.mixers[i]
        if isinstance(m, GatedAttention):
            return m(h, state[0], state[1], pos, self.cos, self.sin)
        return m(h, pos, state[0], state[1])

    def mlp(self, i, h):
        return F.linear(silu_mul(F.linear(h, self.gate_up[i].weight)), self.down[i].weight)

    def layer(self, i, x, state, pos, with_mixer=False):
        """One decoder layer on x [B, T, hidden] at positions [pos, pos + T).  ``with_mixer``: also return
        the mixer's (attention or gated-DeltaNet) output before the residual add."""
        c = self.cfg
        h = self.mixer(i, rms_norm(x, self.norm1[i], c.eps), state, pos)
        x2, n2 = rms_norm(x, self.norm2[i], c.eps, residual=h)
        y = x2 + self.mlp(i, n2)
        return (y, h) if with_mixer else y

    @torch.no_grad()
    def forward_tokens(self, ids, state, pos):
        """ids [B, T] at positions [pos, pos + T) -> logits of the last position [B, vocab].  The
        residual adds ride on the next norm (one ``anemll_rmsnorm`` per add + norm)."""
        c = self.cfg
        x = self.embed(ids)
        h = rms_norm(x, self.norm1[0], c.eps)
        for i in range(c.n_layers):
            x, h = rms_norm(x, self.norm2[i], c.eps, residual=self.mixer(i, h, state[i], pos))
            nxt = self.norm1[i + 1] if i + 1 < c.n_layers else self.norm
            d = self.mlp(i, h)
            if i + 1 < c.n_layers:
                x, h = rms_norm(x, nxt, c.eps, residual=d)
            else:  # the final norm: last position only
                _, h = rms_norm(x[:, -1], nxt, c.eps, residual=d[:, -1])
        return F.linear(h, self.lm_head.weight)

    @torch.no_grad()
    def generate(self, prompt, n_steps, gather=None, graphs=False):
        """Greedy decoding of ``prompt [B, T]``: see :class:`GreedyDecoder` (a fresh one per call)."""
        return GreedyDecoder(self, prompt.shape[0], graphs=graphs)(prompt, n_steps, gather)


class GreedyDecoder:
    """Greedy generation for a fixed batch over one persistent per-sequence state.

    ``decoder(prompt [B, T], n_steps)`` prefills the prompt (one pass per layer over all B*T tokens,
    eager), then runs ``n_steps`` single-token steps and returns the generated ids [B, n_steps + 1]
    (the first from the prefill).  With ``graphs`` each decode position's step -- embedding, 24
    layers, final norm, LM head, argmax, written back into the step's input buffer -- is captured as
    a CUDA graph the first time that position runs (after an eager run of it) and replayed from then
    on; the cache position is a launch argument of the attention kernels, hence one graph per
    position.  The graphs share one memory pool and bake in the state's tensors, which every call
    overwrites from the prefill onwards (rows past the prompt are written before they are read).
    ``gather`` (optional) maps this shard's ids [B] to the job's ids after every step (the NCCL
    all-gather of the next-token ids across ranks); the returned ids are then the job's.
    """

    def __init__(self, model: HybridStack, batch, graphs=True):
        self.model, self.batch, self.use_graphs = model, batch, graphs
        dev = model.lm_head.weight.device
        self.state = model.new_state(batch)
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        self.graphs = {}
        self.pool = None
        self.launches = {}  # library kernel launches of the last eager prefill ("prefill") and of each position

    def _run(self, pos):
        logits = self.model.forward_tokens(self.ids, self.state, pos)
        self.ids.copy_(logits.argmax(-1, keepdim=True))

    def step(self, pos):
        g = self.graphs.get(pos)
        if g is not None:
            g.replay()
            return
        c0 = _lib.launch_count()
        self._run(pos)
        self.launches[pos] = _lib.launch_count() - c0
        if self.use_graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool):
                self._run(pos)
            self.pool = g.pool()
            self.graphs[pos] = g

    @torch.no_grad()
    def prefill(self, prompt):
        """Prefill ``prompt [B, T]`` from position 0; the next-token ids [B] (also kept for the steps)."""
        B, T = prompt.shape
        if B != self.batch:
            raise ValueError(f"decoder built for batch {self.batch}, got {B}")
        if T > self.model.cfg.ctx:
            raise ValueError(f"prompt {T} exceeds the context {self.model.cfg.ctx}")
        c0 = _lib.launch_count()
        self.ids.copy_(self.model.forward_tokens(prompt, self.state, 0).argmax(-1, keepdim=True))
        self.launches["prefill"] = _lib.launch_count() - c0
        return self.ids.view(-1)

    @torch.no_grad()
    def decode(self, pos, n_steps, gather=None):
        """``n_steps`` greedy steps at positions [pos, pos + n_steps); the ids of every step."""
        if pos + n_steps > self.model.cfg.ctx:
            raise ValueError(f"positions up to {pos + n_steps} exceed the context {self.model.cfg.ctx}")
        out = []
        for s in range(n_steps):
            self.step(pos + s)
            out.append(gather(self.ids.view(-1)) if gather else self.ids.view(-1).clone())
        return out

    @torch.no_grad()
    def __call__(self, prompt, n_steps, gather=None):
        T = prompt.shape[1]
        if T + n_steps > self.model.cfg.ctx:
            raise ValueError(f"prompt {T} + {n_steps} steps exceed the context {self.model.cfg.ctx}")
        first = self.prefill(prompt)
        out = [gather(first) if gather else first.clone()] + self.decode(T, n_steps, gather)
        return torch.stack(out, dim=1)


def nccl_id_gather(group=None):
    """``gather`` for :class:`GreedyDecoder` under torch.distributed: every rank holds an equal shard of
    the job's sequences (rank r owns sequences [r*B, (r+1)*B)); returns the job's ids [world*B]."""
    import torch.distributed as dist
    ws = dist.get_world_size(group)

    def gather(ids):
        out = torch.empty(ws * ids.numel(), dtype=ids.dtype, device=ids.device)
        dist.all_gather_into_tensor(out, ids.contiguous(), group=group)
        return out
    return gather


def shard(total, rank, world):
    """This rank's slice [lo, hi) of ``total`` sequences split evenly over ``world`` ranks."""
    if total % world:
        raise ValueError(f"{total} sequences do not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per
