"""The gpt-oss-20b-shaped decoder of benchmark config 2 (cache_eviction_b200.oss20b)
on a small configuration of the same architecture (4 layers alternating a
16-token sliding window and full attention, 64 query / 8 KV heads of 64,
hidden 256, 8 SwiGLU experts top 2, vocabulary 1,000), against a plain
torch fp32 restatement of the same math: per step, the logits of a prompt fed
through the decoder and of greedy steps after it, with the decoder's own
tokens fed to the restatement (so a near-tie cannot make them diverge).  Both
the eager step and the CUDA-graph step; the ring of the sliding-window layers
wraps.  The batch-1 expert GEMVs (ce_moe_gate_up / ce_moe_down) are also
checked on their own against torch.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from cache_eviction_b200 import capi
    capi.load()


def test_moe_gemvs_match_torch():
    from cache_eviction_b200 import oss20b
    gen = torch.Generator(device=DEV).manual_seed(3)
    E, I, D, K = 32, 2880, 2880, 4
    x = torch.randn((1, D), generator=gen, device=DEV).to(torch.bfloat16)
    w1 = (torch.randn((E, 2 * I, D), generator=gen, device=DEV) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, D, I), generator=gen, device=DEV) * 0.02).to(torch.bfloat16)
    ids = torch.tensor([5, 31, 0, 17], dtype=torch.int32, device=DEV)
    wts = torch.tensor([0.4, 0.3, 0.2, 0.1], device=DEV)
    g = torch.empty((K, I), dtype=torch.bfloat16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    oss20b.moe_gate_up(x, w1, ids, g, err)
    y = x.clone()
    oss20b.moe_down(g, w2, ids, wts, y, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    w1f, w2f, xf = w1.float(), w2.float(), x.float()[0]
    want_g = torch.stack([F.silu(w1f[e, :I] @ xf) * (w1f[e, I:] @ xf) for e in ids.tolist()])
    torch.testing.assert_close(g.float(), want_g, rtol=2e-2, atol=2e-3)
    want_y = xf + sum(wts[k] * (w2f[e] @ g[k].float()) for k, e in enumerate(ids.tolist()))
    torch.testing.assert_close(y.float()[0], want_y, rtol=2e-2, atol=2e-3)


class Restated:
    """The decoder's math in fp32 torch, with every K/V kept."""

    def __init__(self, w, cfg):
        self.w, self.cfg = w, cfg
        self.k = [[] for _ in range(cfg.layers)]
        self.v = [[] for _ in range(cfg.layers)]

    def rope(self, t, pos):
        hd = self.cfg.head_dim
        inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, hd, 2, device=DEV, dtype=torch.float32) / hd))
        ang = pos * inv
        a, b = t[..., 0::2], t[..., 1::2]
        return torch.stack((a * ang.cos() - b * ang.sin(), b * ang.cos() + a * ang.sin()), -1).flatten(-2)

    def step(self, tok, pos):
        cfg, W = self.cfg, self.w
        hd, Hq, G = cfg.head_dim, cfg.q_heads, cfg.kv_heads
        bf = lambda t: t.to(torch.bfloat16).float()
        x = W.embed[tok].float()
        for l in range(cfg.layers):
            lw = W.layers[l]
            h = bf(F.rms_norm(x, (cfg.hidden,), lw["ln1"].float(), 1e-5))
            qkv = bf(h @ lw["wqkv"].float() + lw["bqkv"].float())
            q = bf(self.rope(qkv[:Hq * hd].view(Hq, hd), pos))
            k = bf(self.rope(qkv[Hq * hd:(Hq + G) * hd].view(G, hd), pos))
            v = qkv[(Hq + G) * hd:].view(G, hd)
            self.k[l].append(k)
            self.v[l].append(v)
            ks, vs = torch.stack(self.k[l]), torch.stack(self.v[l])      # [T, G, hd]
            if not cfg.full_layer(l):
                ks, vs = ks[-cfg.window:], vs[-cfg.window:]
            qg = q.view(G, Hq // G, hd)
            s = torch.einsum("gjd,tgd->gjt", qg, ks) * hd ** -0.5
            sink = lw["sinks"].view(G, Hq // G, 1)
            p = torch.softmax(torch.cat((s, sink), -1), -1)[..., :-1]
            o = bf(torch.einsum("gjt,tgd->gjd", p, vs).reshape(-1))
            x = bf(x + o @ lw["wo"].float())
            h = bf(F.rms_norm(x, (cfg.hidden,), lw["ln2"].float(), 1e-5))
            r = bf(h @ lw["wr"].float() + lw["br"].float())     # the router's logits are bf16
            tv, ti = torch.topk(r, cfg.top_k)
            wts = torch.softmax(tv, 0)
            y = torch.zeros_like(x)
            for kk, e in enumerate(ti.tolist()):
                w1, w2 = lw["w1"][e].float(), lw["w2"][e].float()
                gte = bf(F.silu(w1[:cfg.inter] @ h) * (w1[cfg.inter:] @ h))
                y = y + wts[kk] * (w2 @ gte)
            x = bf(x + y)
        h = bf(F.rms_norm(x, (cfg.hidden,), W.ln_f.float(), 1e-5))
        return h @ W.lm_head.float().t()


@pytest.mark.parametrize("graph", [False, True])
def test_small_decoder_matches_restatement(graph):
    from cache_eviction_b200 import oss20b
    cfg = oss20b.OssConfig(layers=4, hidden=256, experts=8, top_k=2, inter=128, vocab=1000, window=16)
    w = oss20b.OssWeights(cfg, DEV, seed=5)
    dec = oss20b.OssDecoder(w, None, max_len=256)
    ref = Restated(w, cfg)
    prompt = torch.randint(0, cfg.vocab, (20,), generator=torch.Generator().manual_seed(6)).to(DEV)
    dec.tok.copy_(prompt[:1])
    steps = 44
    for i in range(steps):
        tok = int(dec.tok.item())
        if graph and i == 2:
            dec.capture()
        nxt = prompt[i + 1:i + 2] if i + 1 < prompt.numel() else None
        dec.step(nxt)
        torch.cuda.synchronize()
        want = ref.step(tok, i)
        got = dec.logits.float()[0]
        rel = float((got - want).norm() / want.norm())
        assert rel < 3e-2, (i, rel)
    assert int(dec.err.item()) == 0
    assert dec.n == steps
