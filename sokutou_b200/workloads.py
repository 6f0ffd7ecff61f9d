"""Seeded synthetic workloads with the shapes of the BASELINE configs (0-based c0..c4).

No model weights or datasets exist here; the seed fixes every value.
  c0  one v4.1-Small-class DiT attention layer, CPU fp32: B=3, H=12, hd=64, L=256, text 64, speaker 192.
  c1  the same attention over a full synthesis on 1 B200, bf16: 12 layers x 20 steps, B=3 on the
      first 10 steps (CFG), B=1 on the rest; L in {128, 256, 512}.
  c2  v4-Large-class: B=3, H=16, hd=128, L=512, text 128, speaker 384; 24 layers x 20 steps.
  c3  Qwen3-TTS-1.7B-class talker decode: 28 layers, 16 q / 8 kv heads, hd 128, 96-token prompt,
      decode to T=1120.
  c4  serving sweep: 32 c2-shaped DiT syntheses with L ~ U[96,384] and 32 c3-shaped decodes with
      final T ~ U[200,1500].
Values: q/k/v projections ~ N(0,1)·sigma (sigma = 1/8 for c0/c1, 1/sqrt(hd) for c2); the q/k
producer then applies QK-RMSNorm (weights 1) and RoPE (theta 1e4) as the engine does; the
conditioning keys are drawn already normalised (unit RMS per head), as the engine's ctx K arrive
k-normed (engine/fast.py:278-285). Text valid length ~ U[16, 64] (c2: U[16, 128]).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class DitShape:
    name: str
    H: int
    hd: int
    L: int
    Tb: int
    Sp: int
    n_layers: int
    n_steps: int = 20
    n_cfg_steps: int = 10
    sigma: float = 1 / 8
    text_lo: int = 16
    text_hi: int = 64

    @property
    def S(self) -> int:
        return self.Tb + self.Sp

    @property
    def K(self) -> int:
        return self.L + self.S

    def flops(self, B: int) -> int:
        """4·B·H·L·K·hd per call (every key handed to the kernel, masked ones included)."""
        return 4 * B * self.H * self.L * self.K * self.hd

    def synthesis_calls(self) -> list[int]:
        """Batch size of every attention call of one synthesis, in order."""
        return [3 if s < self.n_cfg_steps else 1 for s in range(self.n_steps) for _ in range(self.n_layers)]

    def synthesis_flops(self) -> int:
        return sum(self.flops(B) for B in self.synthesis_calls())


C0 = DitShape("c0", H=12, hd=64, L=256, Tb=64, Sp=192, n_layers=1, n_steps=1, n_cfg_steps=1)


def c1(L: int) -> DitShape:
    return DitShape(f"c1_L{L}", H=12, hd=64, L=L, Tb=64, Sp=192, n_layers=12)


C1_SWEEP = (128, 256, 512)
C2 = DitShape("c2", H=16, hd=128, L=512, Tb=128, Sp=384, n_layers=24, sigma=1 / math.sqrt(128), text_hi=128)


C4_L_MAX = 384  # the largest latent length of a c4 DiT request (L ~ U[96, 384])


def c4_dit(L: int) -> DitShape:
    return DitShape(f"c4_L{L}", H=16, hd=128, L=L, Tb=128, Sp=384, n_layers=24, sigma=1 / math.sqrt(128), text_hi=128)


@dataclass(frozen=True)
class DecodeShape:
    name: str = "c3"
    n_layers: int = 28
    nq: int = 16
    nkv: int = 8
    hd: int = 128
    prompt: int = 96
    T_final: int = 1120
    theta: float = 1e6
    eps: float = 1e-6
    hidden: int = 256      # synthetic talker width (the GEMVs around the attention are stand-ins)
    vocab: int = 2048

    def layer_bytes(self, T: int, elem: int = 2) -> int:
        """Algorithmic bytes of one layer's decode attention at T keys: K+V read, K/V append, qkv in, out."""
        return (2 * self.nkv * T * self.hd * elem + 2 * self.nkv * self.hd * elem
                + (self.nq + 2 * self.nkv) * self.hd * 4 + self.nq * self.hd * 4)

    def decode_bytes(self, elem: int = 2) -> int:
        return sum(self.layer_bytes(T, elem) * self.n_layers for T in range(self.prompt + 1, self.T_final + 1))


C3 = DecodeShape()


def _norm_heads(x: torch.Tensor) -> torch.Tensor:
    return x * torch.rsqrt((x.float() ** 2).mean(-1, keepdim=True) + 1e-6).to(x.dtype)


def dit_call_inputs(shape: DitShape, B: int, seed: int, device="cpu", dtype=torch.float32):
    """One attention call's raw inputs, drawn in the order q_lat, k_lat, v_lat, k_text, v_text, k_spk,
    v_spk, then the text valid length:
      o4     (B*L, 4*H*hd): [q | k | v | gate] rows for the producer
      ctx_k, ctx_v (S, H, hd): text then speaker keys/values (keys unit-RMS per head)
      bias3  (3, K) additive CFG bias (row 0 alone for B=1)
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    H, hd, L = shape.H, shape.hd, shape.L
    D = H * hd
    sig = shape.sigma
    q = torch.randn(B, L, D, generator=g) * sig
    k = torch.randn(B, L, D, generator=g) * sig
    v = torch.randn(B, L, D, generator=g) * sig
    k_text = torch.randn(shape.Tb, H, hd, generator=g)
    v_text = torch.randn(shape.Tb, H, hd, generator=g) * sig
    k_spk = torch.randn(shape.Sp, H, hd, generator=g)
    v_spk = torch.randn(shape.Sp, H, hd, generator=g) * sig
    n_text = int(torch.randint(shape.text_lo, shape.text_hi + 1, (1,), generator=g))
    gate = torch.zeros(B, L, D)
    o4 = torch.cat([q, k, v, gate], dim=-1).reshape(B * L, 4 * D)
    ctx_k = _norm_heads(torch.cat([k_text, k_spk]))
    ctx_v = torch.cat([v_text, v_spk])
    from .dit import cfg_bias
    bias3 = cfg_bias(L, shape.Tb, shape.Sp, L, n_text, dtype=torch.float32)
    cast = lambda t: t.to(device=device, dtype=dtype).contiguous()
    return {"o4": cast(o4), "ctx_k": cast(ctx_k), "ctx_v": cast(ctx_v), "bias3": cast(bias3), "n_text": n_text}


def dit_qk_weights(shape: DitShape, device="cpu") -> torch.Tensor:
    """QK-RMSNorm weights (2, H, hd) = 1."""
    return torch.ones((2, shape.H, shape.hd), dtype=torch.float32, device=device)


def dit_freqs(n_pos: int, hd: int, theta: float = 1e4, device="cpu") -> torch.Tensor:
    """(n_pos, hd/2, 2) float32 (cos, sin) RoPE table of the latent positions."""
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = torch.arange(n_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.stack([ang.cos(), ang.sin()], dim=-1).float().to(device).contiguous()


def serving_requests(seed: int = 0, n_dit: int = 32, n_decode: int = 32):
    """The c4 request list: [(kind, size)] with kind 'dit' (size = latent length L ~ U[96,384]) or
    'decode' (size = final KV length T ~ U[200,1500]), interleaved in a seeded order."""
    g = torch.Generator().manual_seed(seed)
    dit = [("dit", int(x)) for x in torch.randint(96, C4_L_MAX + 1, (n_dit,), generator=g)]
    dec = [("decode", int(x)) for x in torch.randint(200, 1501, (n_decode,), generator=g)]
    order = torch.randperm(n_dit + n_decode, generator=g).tolist()
    reqs = dit + dec
    return [reqs[i] for i in order]


class SyntheticTalker:
    """A seeded stand-in for the Qwen3 talker stack around the decode attention (c3).

    Per position: h = input row; for each layer h += W_o · attn(W_qkv · rmsnorm(h)); the greedy
    token is argmax(W_out · rmsnorm(h)); the next position's input is that token's embedding.
    Weights ~ N(0, 1/fan_in); qn, kn ~ 1 + N(0, 0.02). Only the attention is the product's kernel:
    the projections are torch fp32 matmuls standing in for the engine's GEMVs.
    """

    def __init__(self, shape: DecodeShape = C3, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        s = shape
        Dq = (s.nq + 2 * s.nkv) * s.hd
        self.shape = s
        self.w = {
            "prompt": torch.randn(s.prompt, s.hidden, generator=g),
            "emb": torch.randn(s.vocab, s.hidden, generator=g),
            "w_qkv": torch.randn(s.n_layers, Dq, s.hidden, generator=g) / math.sqrt(s.hidden),
            "w_o": torch.randn(s.n_layers, s.hidden, s.nq * s.hd, generator=g) / math.sqrt(s.nq * s.hd),
            "qn": 1 + 0.02 * torch.randn(s.n_layers, s.hd, generator=g),
            "kn": 1 + 0.02 * torch.randn(s.n_layers, s.hd, generator=g),
            "w_out": torch.randn(s.vocab, s.hidden, generator=g) / math.sqrt(s.hidden),
        }

    def numpy_weights(self) -> dict:
        return {k: v.numpy() for k, v in self.w.items()}

    @torch.no_grad()
    def generate(self, device, n_new: int, cache_dtype: torch.dtype = torch.float32, max_len: int | None = None,
                 fused: bool = False):
        """Greedy tokens of positions prompt-1 .. prompt-1+n_new through the B200 decode attention; with
        fused=True every layer's rms_gemv(qkv) -> attention -> gemv(o) runs as the one-launch block kernel
        (input RMSNorm weight 1, fp32 weights) instead of torch projections around the attention."""
        from .qwen3 import TalkerAttention

        s = self.shape
        w = {k: v.to(device) for k, v in self.w.items()}
        max_len = max_len or (s.prompt + n_new)
        ta = TalkerAttention(s.n_layers, s.nq, s.nkv, max_len, s.theta, s.eps, device, cache_dtype, s.hd)
        att = torch.empty(s.nq * s.hd, device=device)
        ones = torch.ones(s.hidden, device=device)
        rms = lambda h: h * torch.rsqrt((h * h).mean() + s.eps)
        tokens = []
        tok = None
        for pos in range(s.prompt + n_new):
            h = w["prompt"][pos] if pos < s.prompt else w["emb"][tok]
            if fused:
                h = h.clone()
            for li in range(s.n_layers):
                if fused:
                    ta.block(li, h, ones, s.eps, w["w_qkv"][li], w["qn"][li], w["kn"][li], w["w_o"][li])
                    continue
                qkv = (w["w_qkv"][li] @ rms(h)).contiguous()
                ta.attn(li, qkv, w["qn"][li], w["kn"][li], att)
                h = h + w["w_o"][li] @ att
            if pos >= s.prompt - 1:
                tok = int(torch.argmax(w["w_out"] @ rms(h)))
                tokens.append(tok)
            ta.pos.add_(1)
        return tokens, ta
