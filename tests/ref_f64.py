"""An independent float64 forward of the Qwen3/Llama decoder (transformers' modeling_qwen3
semantics: RMSNorm, q/k norms, RoPE rotate_half, GQA softmax attention, SwiGLU), used only to
check the oracle's structure, as the reference's own qwen3_test.go:80-205 checks milcpu against a
float64 restatement."""

import numpy as np

from hwnpu_b200 import synth


def dequant(lin):
    import ctypes as C
    import oracle_lib as O

    out = np.empty(lin.rows * lin.cols, np.float32)
    L = O.lib()
    u8, u16, f32 = O._u8p, O._u16p, O._f32p
    from hwnpu_b200 import _abi as A
    if lin.fmt == A.HC_FMT_INT8_ROW:
        L.or_dequant_linear(O.p(lin.data, u8), O.p(lin.scales, u16), lin.rows, lin.cols, lin.cols, 8, O.p(out, f32))
    elif lin.fmt == A.HC_FMT_INT4_SYM_G32:
        L.or_dequant_linear(O.p(lin.data, u8), O.p(lin.scales, u16), lin.rows, lin.cols, 32, 4, O.p(out, f32))
    elif lin.fmt == A.HC_FMT_INT4_ASYM_G32:
        L.or_dequant_int4_asym(O.p(lin.data, u8), O.p(lin.scales, u16), O.p(lin.zeros, u16), lin.rows, lin.cols, O.p(out, f32))
    else:
        for r in range(lin.rows):
            L.or_mxfp4_dequant(O.p(lin.data[r * lin.cols // 2:], u8), O.p(lin.exps[r * lin.cols // 32:], u8), lin.cols, O.p(out[r * lin.cols:], f32))
    return out.reshape(lin.rows, lin.cols).astype(np.float64)


def rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def forward(model, tokens):
    """Logits (float64, [len(tokens)][vocab]) of a causal pass over tokens from position 0."""
    c = model.cfg
    hd, H, KV = c.head_dim, c.heads, c.kv_heads
    n = len(tokens)
    if c.tied:
        E = dequant(model.head)
        x = synth.f16_values(synth.f16_bits(E[tokens].astype(np.float32))).astype(np.float64)
    else:
        x = synth.f16_values(model.embed.reshape(c.vocab, c.hidden)[tokens]).astype(np.float64)
    inv = 1.0 / c.rope_theta ** (np.arange(0, hd, 2) / hd)
    ang = np.arange(n)[:, None] * inv[None, :]
    cos = np.concatenate([np.cos(ang)] * 2, -1)
    sin = np.concatenate([np.sin(ang)] * 2, -1)

    def rope(t):  # [n, heads, hd]
        rot = np.concatenate([-t[..., hd // 2:], t[..., :hd // 2]], -1)
        return t * cos[:, None, :] + rot * sin[:, None, :]

    f = lambda h: synth.f16_values(h).astype(np.float64)
    for L in model.layers:
        h = rms(x, f(L["input_norm"]), c.norm_eps)
        q = (h @ dequant(L["q"]).T).reshape(n, H, hd)
        k = (h @ dequant(L["k"]).T).reshape(n, KV, hd)
        v = (h @ dequant(L["v"]).T).reshape(n, KV, hd)
        if c.qk_norm:
            q = rms(q, f(L["q_norm"]), c.norm_eps)
            k = rms(k, f(L["k_norm"]), c.norm_eps)
        q, k = rope(q), rope(k)
        rep = H // KV
        o = np.zeros((n, H, hd))
        mask = np.triu(np.full((n, n), -np.inf), 1)
        for hh in range(H):
            s = q[:, hh] @ k[:, hh // rep].T / np.sqrt(hd) + mask
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            o[:, hh] = p @ v[:, hh // rep]
        x = x + o.reshape(n, H * hd) @ dequant(L["o"]).T
        h = rms(x, f(L["post_norm"]), c.norm_eps)
        g = h @ dequant(L["gate"]).T
        u = h @ dequant(L["up"]).T
        x = x + (g / (1 + np.exp(-g)) * u) @ dequant(L["down"]).T
    h = rms(x, f(model.final_norm), c.norm_eps)
    return h @ dequant(model.head).T
