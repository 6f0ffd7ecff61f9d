"""Generate the golden fixtures under tests/golden/ from the reference's own code.

Run in the container that holds the sokutou reference checkout (it is NOT needed at test time):

    python tests/golden/make_golden.py --reference <path to the sokutou checkout>

What it runs, and why it pins the CPU oracle:

* DiT attention (`dit_*.npz`): the reference's exact-math DiT core `engine.fast.DitCore`
  (engine/fast.py:97-185) on a small random model, with `cudnn_attention = False` as the bucketed
  engine sets it (engine/bucket.py:92), so attention goes through
  `F.scaled_dot_product_attention` (engine/fast.py:169-171). The script records, for every layer,
  the fused projection output `o` (engine/fast.py:156), the q/k/v/mask handed to SDPA and the SDPA
  output. The key masks come from the reference's own `BucketSampler._fill` and
  `FusedBucketSampler._fill` (engine/bucket.py:240-259, engine/fused.py:373-378).
  The reference imports the third-party package `irodori_tts` at module top (engine/fast.py:41-44);
  it is absent here, so the four names it imports are stubbed with placeholders that the recorded
  code never calls (`DitCore` and `_fill` use none of them).
* Decode attention (`decode_*.npz`): the Qwen3 attention functions of transformers 5.5.0
  (`Qwen3RMSNorm`, `Qwen3RotaryEmbedding`, `apply_rotary_pos_emb`, `eager_attention_forward`),
  which the reference's `attn` kernel (qwen3/kernels.py:338-414) reproduces for the qwen-tts
  talker, applied to one decode step over a bf16 (or fp32) cache.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _stub_irodori():
    """Placeholders for `irodori_tts` so that engine/fast.py, bucket.py and fused.py import."""
    def _unavailable(*a, **k):
        raise RuntimeError("irodori_tts is not installed; this stub must not be called")

    pkg = types.ModuleType("irodori_tts")
    mods = {
        "irodori_tts.model": {},
        "irodori_tts.attention": {"masked_sdpa": _unavailable},
        "irodori_tts.meanflow": {"sample_euler_meanflow": _unavailable},
        "irodori_tts.rf": {"draw_initial_noise": _unavailable, "sample_euler_rf_cfg": _unavailable},
    }
    sys.modules["irodori_tts"] = pkg
    for name, attrs in mods.items():
        m = types.ModuleType(name)
        for k, v in attrs.items():
            setattr(m, k, v)
        sys.modules[name] = m
        setattr(pkg, name.split(".")[1], m)


class _Norm:
    def __init__(self, w, eps):
        self.weight, self.eps = w, eps


def _fake_dit(H, hd, n_layers, hidden, g):
    """An object with the attributes DitCore.__init__ reads (engine/fast.py:108-129)."""
    dim = H * hd
    lin = lambda o, i: torch.nn.Linear(i, o, bias=False)
    blocks = []
    for _ in range(n_layers):
        att = types.SimpleNamespace(heads=H, head_dim=hd, dim=dim,
                                    wq=lin(dim, dim), wk=lin(dim, dim), wv=lin(dim, dim), gate=lin(dim, dim),
                                    wo=lin(dim, dim),
                                    q_norm=_Norm(1 + 0.1 * torch.randn(H, hd, generator=g), 1e-6),
                                    k_norm=_Norm(1 + 0.1 * torch.randn(H, hd, generator=g), 1e-6))
        mlp = types.SimpleNamespace(w1=lin(hidden, dim), w3=lin(hidden, dim), w2=lin(dim, hidden))
        blocks.append(types.SimpleNamespace(attention=att, mlp=mlp,
                                            attention_adaln=types.SimpleNamespace(eps=1e-6),
                                            mlp_adaln=types.SimpleNamespace(eps=1e-6)))
    model = types.SimpleNamespace(in_proj=lin(dim, 32), out_norm=torch.nn.Identity(), out_proj=lin(32, dim),
                                  blocks=blocks, dtype=torch.float32, device=torch.device("cpu"))
    return model


def _ref_bias(fused, bucket, lb, tb, n_spk, seq_len, n_text, H, hd):
    """bias3 exactly as FusedBucketSampler._fill builds it (engine/fused.py:373-378)."""
    self = object.__new__(fused.FusedBucketSampler)
    self.device, self.wdtype = torch.device("cpu"), torch.float32
    self._bias_bufs, self._recording = {}, None
    ctx = types.SimpleNamespace(tb=tb, k=torch.zeros(1, 1, tb + n_spk, H, hd), v=torch.zeros(1, 1, tb + n_spk, H, hd),
                                voice=None)
    sh = types.SimpleNamespace(lb=lb, tb=tb, n_spk=n_spk, ctx=ctx, filled=None,
                               mask3=torch.ones((3, 1, 1, lb + tb + n_spk), dtype=torch.bool))
    voice = types.SimpleNamespace(kv=[(torch.zeros(1, n_spk, H, hd), torch.zeros(1, n_spk, H, hd))])
    tk = torch.zeros(1, 1, n_text, H, hd)
    fused.FusedBucketSampler._fill(self, sh, seq_len, n_text, voice, tk, tk)
    return sh.mask3.reshape(3, -1).numpy().copy(), sh.bias3.reshape(3, -1).numpy().copy()


def make_dit(ref_root):
    sys.path.insert(0, ref_root)
    _stub_irodori()
    import engine.bucket as bucket  # noqa: F401  (reference module)
    import engine.fast as fast      # reference module
    import engine.fused as fused    # reference module
    import torch.nn.functional as F

    out = {}
    for case, (H, hd, L, Tb, n_text, Sp, n_layers, seed) in {
        "dit_small": (4, 64, 20, 8, 5, 12, 2, 1),
        "dit_hd128": (2, 128, 33, 16, 16, 7, 2, 2),
    }.items():
        g = torch.Generator().manual_seed(seed)
        torch.manual_seed(seed)
        model = _fake_dit(H, hd, n_layers, 2 * H * hd, g)
        core = fast.DitCore(model, torch.float32)
        core.cudnn_attention = False                     # engine/bucket.py:92 default
        dim = H * hd
        B = 3
        lb = L                                           # no latent padding: seq_len = lb - 3 below
        seq_len = L - 3
        mask3, bias3 = _ref_bias(fused, bucket, lb, Tb, Sp, seq_len, n_text, H, hd)
        x = torch.randn(1, lb, 32, generator=g)
        coef = torch.randn(n_layers, 6, 1, 1, dim, generator=g) * 0.3 + torch.tensor([1, 0, 1, 1, 0, 1.0]).reshape(1, 6, 1, 1, 1)
        ctx_k = torch.randn(n_layers, 1, Tb + Sp, H, hd, generator=g)
        ctx_v = torch.randn(n_layers, 1, Tb + Sp, H, hd, generator=g)
        ang = torch.arange(lb, dtype=torch.float64)[:, None] * (1e4 ** (-torch.arange(0, hd, 2, dtype=torch.float64) / hd))
        freqs_c = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)[None, :, None, None, :]
        rec = {"o": [], "sdpa": [], "gated": []}
        orig_linear, orig_sdpa = F.linear, F.scaled_dot_product_attention
        wq = {id(p["w_qkvg"]) for p in core.layers}
        wo = {id(p["w_o"]) for p in core.layers}

        def linear(x_, w, b=None):
            y = orig_linear(x_, w, b)
            if id(w) in wq:
                rec["o"].append(y.detach().clone())
            if id(w) in wo:                               # input of w_o = y · sigmoid(gate)
                rec["gated"].append(x_.detach().clone())
            return y

        def sdpa(q, k, v, attn_mask=None, **kw):
            y = orig_sdpa(q, k, v, attn_mask=attn_mask, **kw)
            rec["sdpa"].append((q.detach().clone(), k.detach().clone(), v.detach().clone(),
                                attn_mask.detach().clone(), y.detach().clone()))
            return y

        F.linear, F.scaled_dot_product_attention = linear, sdpa
        try:
            with torch.no_grad():
                core(x.expand(3, -1, -1), coef, ctx_k, ctx_v, torch.from_numpy(mask3).reshape(3, 1, 1, -1), freqs_c)
        finally:
            F.linear, F.scaled_dot_product_attention = orig_linear, orig_sdpa
        li = n_layers - 1                                 # last layer: batch rows differ
        q, k, v, m, y = rec["sdpa"][li]
        o = rec["o"][li].reshape(B * lb, 4 * dim)
        qk_w = torch.stack([model.blocks[li].attention.q_norm.weight, model.blocks[li].attention.k_norm.weight])
        out[case] = dict(
            H=H, hd=hd, L=lb, Tb=Tb, Sp=Sp, n_text=n_text, seq_len=seq_len, qk_eps=1e-6,
            o4=o.numpy(), qk_w=qk_w.float().numpy(),
            freqs=torch.view_as_real(freqs_c[0, :, 0, 0, :]).numpy(),
            ctx_k=ctx_k[li, 0].numpy(), ctx_v=ctx_v[li, 0].numpy(),
            q=q.contiguous().numpy(), k=k.contiguous().numpy(),           # as SDPA receives them: (B, H, *, hd)
            v=v.contiguous().numpy(), mask=m.reshape(B, -1).numpy(),
            y=y.transpose(1, 2).contiguous().numpy(),     # (B, L, H, hd)
            gated=rec["gated"][li].reshape(B * lb, dim).numpy(),  # engine/fast.py:174, the `gate` output
            mask3=mask3, bias3=bias3,
        )
    # Extra mask cases (padding in every segment, single text token, full text bucket).
    masks = {}
    for i, (lb, tb, ns, sl, nt) in enumerate([(24, 8, 12, 20, 5), (16, 24, 10, 16, 24), (32, 64, 50, 29, 1),
                                              (128, 64, 192, 100, 37)]):
        m3, b3 = _ref_bias(fused, bucket, lb, tb, ns, sl, nt, 2, 8)
        masks[f"case{i}"] = dict(lb=lb, tb=tb, n_spk=ns, seq_len=sl, n_text=nt, mask3=m3, bias3=b3)
    return out, masks


def make_decode():
    from transformers import Qwen3Config
    from transformers.models.qwen3 import modeling_qwen3 as mq

    out = {}
    for case, (nq, nkv, T, max_len, cache, theta, seed) in {
        "decode_bf16": (4, 2, 37, 48, "bf16", 1e6, 3),
        "decode_f32": (4, 2, 70, 80, "f32", 1e6, 4),
        "decode_cp": (4, 2, 5, 16, "bf16", 1e6, 5),
    }.items():
        hd = 128
        g = torch.Generator().manual_seed(seed)
        cfg = Qwen3Config(hidden_size=nq * hd, num_attention_heads=nq, num_key_value_heads=nkv, head_dim=hd,
                          max_position_embeddings=max_len, rope_parameters={"rope_type": "default", "rope_theta": theta})
        rot = mq.Qwen3RotaryEmbedding(cfg)
        qn_m, kn_m = mq.Qwen3RMSNorm(hd, eps=1e-6), mq.Qwen3RMSNorm(hd, eps=1e-6)
        with torch.no_grad():
            qn_m.weight.copy_(1 + 0.02 * torch.randn(hd, generator=g))
            kn_m.weight.copy_(1 + 0.02 * torch.randn(hd, generator=g))
        pos = T - 1
        cdt = torch.bfloat16 if cache == "bf16" else torch.float32
        Kc = torch.randn(nkv, max_len, hd, generator=g).to(cdt)
        Vc = torch.randn(nkv, max_len, hd, generator=g).to(cdt)
        Kc0, Vc0 = Kc.clone(), Vc.clone()
        qkv = torch.randn((nq + 2 * nkv) * hd, generator=g)
        q = qkv[: nq * hd].view(1, 1, nq, hd)
        k = qkv[nq * hd:(nq + nkv) * hd].view(1, 1, nkv, hd)
        v = qkv[(nq + nkv) * hd:].view(1, 1, nkv, hd)
        with torch.no_grad():
            q = qn_m(q).transpose(1, 2)                  # (1, nq, 1, hd)
            k = kn_m(k).transpose(1, 2)
            cos, sin = rot(q, torch.tensor([[pos]]))
            q, k = mq.apply_rotary_pos_emb(q, k, cos, sin)
            Kc[:, pos] = k[0, :, 0].to(cdt)
            Vc[:, pos] = v[0, 0].to(cdt)
            module = types.SimpleNamespace(num_key_value_groups=nq // nkv, training=False)
            att, _ = mq.eager_attention_forward(module, q, Kc[None, :, :T].float(), Vc[None, :, :T].float(), None,
                                                scaling=hd ** -0.5)
            cos_all, sin_all = rot(q, torch.arange(max_len)[None])
        rope = torch.cat([cos_all[0, :, :hd // 2], sin_all[0, :, :hd // 2]], dim=1).contiguous()
        as_store = (lambda t: t.view(torch.int16).numpy().view(np.uint16)) if cache == "bf16" else (lambda t: t.numpy())
        out[case] = dict(nq=nq, nkv=nkv, hd=hd, T=T, pos=pos, max_len=max_len, eps=1e-6, cache=cache,
                         qkv=qkv.numpy(), qn=qn_m.weight.detach().numpy(), kn=kn_m.weight.detach().numpy(),
                         rope=rope.numpy(), Kc0=as_store(Kc0), Vc0=as_store(Vc0),
                         k_row=Kc[:, pos].float().numpy(), v_row=Vc[:, pos].float().numpy(),
                         out=att.reshape(-1).numpy())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the sokutou checkout (contains engine/)")
    a = ap.parse_args()
    dit, masks = make_dit(a.reference)
    for name, d in dit.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
    np.savez_compressed(os.path.join(HERE, "dit_masks.npz"),
                        **{f"{c}_{k}": v for c, d in masks.items() for k, v in d.items()})
    for name, d in make_decode().items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
