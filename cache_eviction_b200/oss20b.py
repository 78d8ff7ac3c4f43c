"""A gpt-oss-20b-shaped decoder with random weights, around the eviction engine.

benchmark config 2: 24 layers alternating a 128-token sliding window (even
layers) and full attention (odd layers), 64 query / 8 KV heads of 64, hidden
2880, attention sinks, a mixture of 32 SwiGLU experts (top 4, width 2880) per
layer and a 201,088-token vocabulary, all bf16 and randomly initialised (no
checkpoint is involved).  Batch 1, greedy decoding.

The reference serves the real model in SGLang with the eviction overlay on
its 12 full-attention layers; the sliding-window layers keep their native
128-token window and are never evicted (code/SGLANG.md:49,
code/modal_server.py:85-89).  Here:

  * full layers: K/V in the RaggedDecodeEngine's paged pools; the fused
    decode attention + H2O score (ce_decode_attn_score) and boundaries every
    2,048 tokens (ce_boundary) are this repository's kernels;
  * sliding-window layers: a 128-slot ring per layer at page size 1, attended
    by the same decode kernel with scoring off;
  * dense projections: cuBLAS through torch; the batch-1 expert GEMVs are
    ce_moe_gate_up / ce_moe_down, which read the router's choice on the
    device, so a whole step (embedding, 24 layers, LM head, argmax) is one
    CUDA graph.  A prompt is fed through the same step, one token at a time.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import capi, kernels
from .engine import RaggedDecodeEngine
from .policy import EvictionConfig


@dataclass(frozen=True)
class OssConfig:
    layers: int = 24
    hidden: int = 2880
    q_heads: int = 64
    kv_heads: int = 8
    head_dim: int = 64
    experts: int = 32
    top_k: int = 4
    inter: int = 2880
    vocab: int = 201088
    window: int = 128
    rope_theta: float = 150000.0

    def full_layer(self, l: int) -> bool:
        return l % 2 == 1


def moe_gate_up(x, w1, ids, g, err=None):
    """g[k] = silu(W1[ids[k], :I] x) * (W1[ids[k], I:] x) (ce_moe_gate_up)."""
    lib = capi.load()
    E, two_i, dim = w1.shape
    st = lib.ce_moe_gate_up(C.c_void_p(x.data_ptr()), C.c_void_p(w1.data_ptr()), C.c_void_p(ids.data_ptr()),
                            int(ids.numel()), E, two_i // 2, dim, C.c_void_p(g.data_ptr()),
                            None if err is None else C.c_void_p(err.data_ptr()),
                            C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    capi.check(st, "ce_moe_gate_up")
    kernels._count(1)


def moe_down(g, w2, ids, weights, x, err=None):
    """x += sum_k weights[k] W2[ids[k]] g[k] (ce_moe_down)."""
    lib = capi.load()
    E, dim, inter = w2.shape
    st = lib.ce_moe_down(C.c_void_p(g.data_ptr()), C.c_void_p(w2.data_ptr()), C.c_void_p(ids.data_ptr()),
                         C.c_void_p(weights.data_ptr()), int(ids.numel()), E, inter, dim, C.c_void_p(x.data_ptr()),
                         None if err is None else C.c_void_p(err.data_ptr()),
                         C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    capi.check(st, "ce_moe_down")
    kernels._count(1)


class OssWeights:
    """Random bf16 weights (uniform with std 0.02; norms at 1; sinks fp32), on the device."""

    def __init__(self, cfg: OssConfig, device, seed: int = 0):
        self.cfg = cfg
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed)
        a = 0.02 * 3 ** 0.5

        def mat(*shape):
            return torch.empty(shape, dtype=torch.bfloat16, device=dev).uniform_(-a, a, generator=gen)

        D, hd = cfg.hidden, cfg.head_dim
        qkv = (cfg.q_heads + 2 * cfg.kv_heads) * hd
        self.embed = mat(cfg.vocab, D)
        self.lm_head = mat(cfg.vocab, D)
        self.ln_f = torch.ones(D, dtype=torch.bfloat16, device=dev)
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append(dict(
                ln1=torch.ones(D, dtype=torch.bfloat16, device=dev),
                ln2=torch.ones(D, dtype=torch.bfloat16, device=dev),
                wqkv=mat(D, qkv), bqkv=mat(qkv), wo=mat(cfg.q_heads * hd, D),
                sinks=torch.randn(cfg.q_heads, generator=gen, device=dev),
                wr=mat(D, cfg.experts), br=mat(cfg.experts),
                w1=mat(cfg.experts, 2 * cfg.inter, D), w2=mat(cfg.experts, D, cfg.inter)))


class OssDecoder:
    """One batch-1 request decoded greedily over shared weights.

    eviction: the policy of the full layers (None: a full cache); scored=False
    keeps the same boundaries with H2O scoring off (the full-cache decode rate
    at the same resident KV)."""

    def __init__(self, weights: OssWeights, eviction: Optional[EvictionConfig], max_len: int,
                 scored: bool = True, device="cuda", page_size: int = 16):
        cfg = weights.cfg
        self.w, self.cfg = weights, cfg
        dev = self.device = torch.device(device)
        self.full = [l for l in range(cfg.layers) if cfg.full_layer(l)]
        P = page_size
        if eviction is not None:
            units = (eviction.budget + 2 * 2048) // P + 64
        else:
            units = -(-max_len // P) + 64
        self.eng = RaggedDecodeEngine(layers=len(self.full), q_heads=cfg.q_heads, kv_heads=cfg.kv_heads,
                                      page_size=P, pool_units=units, max_rows=1,
                                      r2u_width=-(-max_len // P) + 8, pos_cap=max(64, units), device=dev,
                                      boundary_rows=1)
        self.eng.seed_free_units(list(range(1, units)))
        self.eng.add_row(0, eviction, 0)
        if not scored:
            self.eng.mode.fill_(capi.CE_MODE_NONE)
            self.eng.score_flags = 0
        self.eng.commit_rows()
        # the CSR buffer the graph holds must fit the longest row (max_len tokens)
        self.eng._ensure_capacity(max_len)
        nswa = cfg.layers - len(self.full)
        ring = (cfg.window, cfg.kv_heads, 1, cfg.head_dim)
        self.ring_k = [torch.zeros(ring, dtype=torch.bfloat16, device=dev) for _ in range(nswa)]
        self.ring_v = [torch.zeros(ring, dtype=torch.bfloat16, device=dev) for _ in range(nswa)]
        self.swa_indptr = torch.zeros(2, dtype=torch.int32, device=dev)
        self.swa_idx = torch.arange(cfg.window, dtype=torch.int32, device=dev)
        self.swa_ws = torch.empty(kernels.decode_workspace_bytes(1, cfg.window, cfg.q_heads, cfg.kv_heads, 1, 0),
                                  dtype=torch.uint8, device=dev)
        hd = cfg.head_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd))
        ang = torch.arange(max_len + 1, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        self.rot = torch.polar(torch.ones_like(ang), ang)      # e^{i pos theta_j}, complex64
        self.tok = torch.zeros(1, dtype=torch.int64, device=dev)
        self.logits = torch.zeros((1, cfg.vocab), dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros((1, cfg.hidden), dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros((1, cfg.q_heads, hd), dtype=torch.bfloat16, device=dev)
        self.ids = torch.zeros(cfg.top_k, dtype=torch.int32, device=dev)
        self.wts = torch.zeros(cfg.top_k, dtype=torch.float32, device=dev)
        self.g = torch.zeros((cfg.top_k, cfg.inter), dtype=torch.bfloat16, device=dev)
        self.err = self.eng.err
        self.graph = None
        self.scale = hd ** -0.5

    @property
    def n(self) -> int:
        return self.eng.rows[0].n

    # ------------------------------------------------------------ one step
    def _rope(self, qk, rot):
        """Rotary embedding of q and k together: adjacent pairs as complex
        numbers times e^{i pos theta_j}.  qk [1, heads * hd] bf16 view."""
        c = torch.view_as_complex(qk.view(-1, self.cfg.head_dim // 2, 2).float()) * rot
        return torch.view_as_real(c).flatten(-2).to(torch.bfloat16)

    def _device_step(self):
        """Everything of one token on the device: position advance and page
        (engine), CSR, 24 layers, LM head, argmax into self.tok.  Capturable."""
        cfg, W, eng = self.cfg, self.w, self.eng
        hd, Hq, G = cfg.head_dim, cfg.q_heads, cfg.kv_heads
        eng.advance_device()
        eng.fill()
        pos = eng.seq_lens_dev[:1] - 1                        # the new token's position
        rot = self.rot.index_select(0, pos)                   # [1, hd/2] complex
        self.swa_indptr[1:].copy_(torch.clamp(eng.seq_lens_dev[:1], max=cfg.window))
        unit = eng.r2u[0].index_select(0, pos // eng.P).long()
        slot = pos % eng.P
        ring_slot = pos % cfg.window
        self.x.copy_(W.embed.index_select(0, self.tok))
        fi = si = 0
        for l in range(cfg.layers):
            lw = W.layers[l]
            h = F.rms_norm(self.x, (cfg.hidden,), lw["ln1"], 1e-5)
            qkv = torch.addmm(lw["bqkv"], h, lw["wqkv"])
            qk = self._rope(qkv[:, :(Hq + G) * hd], rot)       # [Hq + G, hd]
            q = qk[:Hq].view(1, Hq, hd)
            k = qk[Hq:].view(1, G, hd)
            v = qkv[:, (Hq + G) * hd:].view(1, G, hd)
            if cfg.full_layer(l):
                eng.k[fi][unit, :, slot] = k
                eng.v[fi][unit, :, slot] = v
                eng.decode_layer(fi, q, self.attn, lw["sinks"], self.scale)
                fi += 1
            else:
                self.ring_k[si][ring_slot, :, 0] = k
                self.ring_v[si][ring_slot, :, 0] = v
                kernels.decode_attn_score(q, self.ring_k[si], self.ring_v[si], self.swa_indptr, self.swa_idx, None,
                                          self.scale, 1, sinks=lw["sinks"], out=self.attn, score_flags=0,
                                          err=self.err, workspace=self.swa_ws)
                si += 1
            self.x.addmm_(self.attn.view(1, -1), lw["wo"])
            h = F.rms_norm(self.x, (cfg.hidden,), lw["ln2"], 1e-5)
            top_v, top_i = torch.topk(torch.addmm(lw["br"], h, lw["wr"]), cfg.top_k)
            self.wts.copy_(torch.softmax(top_v[0].float(), 0))
            self.ids.copy_(top_i[0])
            moe_gate_up(h, lw["w1"], self.ids, self.g, self.err)
            moe_down(self.g, lw["w2"], self.ids, self.wts, self.x, self.err)
        h = F.rms_norm(self.x, (cfg.hidden,), W.ln_f, 1e-5)
        torch.matmul(h, W.lm_head.t(), out=self.logits)
        self.tok.copy_(torch.argmax(self.logits, -1))

    def capture(self):
        """Record _device_step as a CUDA graph (after at least one eager step,
        which sizes every workspace)."""
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._device_step()
        torch.cuda.synchronize(self.device)

    def step(self, next_token: Optional[torch.Tensor] = None):
        """Decode one token: the due boundary (eagerly), then the step (the
        graph when captured).  next_token (device int64 [1]) overrides the
        greedy choice, which feeds a prompt through the same path."""
        eng = self.eng
        due = eng.due()
        if due:
            eng.run_boundaries(due)
        eng.advance_host()
        if self.graph is not None:
            self.graph.replay()
        else:
            self._device_step()
        if next_token is not None:
            self.tok.copy_(next_token)

    def prefill(self, prompt: torch.Tensor, eager_steps: int = 2):
        """Feed prompt (device int64 [T]) one token at a time; captures the
        graph after the first eager_steps tokens."""
        self.tok.copy_(prompt[:1])
        for i in range(int(prompt.numel())):
            if i == eager_steps and self.graph is None:
                self.capture()
            nxt = prompt[i + 1:i + 2] if i + 1 < prompt.numel() else None
            self.step(nxt)
