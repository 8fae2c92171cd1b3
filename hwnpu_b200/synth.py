"""Model shapes of the benchmark configurations and their seeded synthetic weights.

The weights are drawn N(0, std^2) per tensor name (hc_synth_normal) and quantised with the
library's converter routines into the reference's byte layouts (palette.QuantizeLinear's int8,
the asymmetric int4 of group 32, MXFP4's Encode), the form hc_model_load takes. A Model keeps
the numpy arrays alive and builds the ctypes descriptor over them.

The generator and the quantisers come from a `gen` object (normal, tokens, quantize, f16_bits);
the default is this package's library (LibGen). A CPU-only caller passes another with the same
results (the oracle's, tests/oracle_lib.OracleGen) so that it never maps libhwnpu_cuda.so.
"""

import ctypes as C
from dataclasses import dataclass, replace

import numpy as np

from . import _abi as A


@dataclass(frozen=True)
class Config:
    name: str
    layers: int
    hidden: int
    inter: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    fmt: int                  # A.HC_FMT_* of every linear layer and the head
    tied: bool = False
    qk_norm: bool = False
    norm_scale: bool = True   # qwen3's normScale 64 (internal/llm/qwen3/build.go:117-151)
    rope_theta: float = 1e4
    norm_eps: float = 1e-6
    std: float = 0.02
    quant_search: bool = False
    # gpt-oss (arch "gptoss"): MXFP4 experts behind a softmax top-k router, bf16 attention, router
    # and head, biases, sinks, sliding layers alternating with full ones (sliding first), YaRN
    arch: str = "qwen3"
    experts: int = 0
    top_k: int = 0
    window: int = 0
    attn_fmt: int = -1        # the attention, router and head format (-1: fmt)
    yarn: tuple = (1.0, 32.0, 1.0, 4096, False)  # factor, beta_fast, beta_slow, original, truncate
    swiglu: tuple = (1.702, 7.0)                  # alpha, limit of gpt-oss's gated unit


# BASELINE.json configs[0] (C1) and configs[1] (C2); C4's draft is C1 with C2's vocabulary.
C1 = Config("c1-llama4L-int8", 4, 1024, 2816, 16, 4, 64, 32000, A.HC_FMT_INT8_ROW)
C2 = Config("c2-qwen3-1.7B-int4g32", 28, 2048, 6144, 16, 8, 128, 151936, A.HC_FMT_INT4_ASYM_G32,
            tied=True, qk_norm=True, rope_theta=1e6)
C4_DRAFT = replace(C1, name="c4-draft-int8", vocab=151936)
# BASELINE.json configs[2] (C3): gpt-oss-20b's shapes (vocabulary 201088, rope theta 150000 with
# YaRN of factor 32 over 4096 positions, rms eps 1e-5, gate limit 7 and alpha 1.702), MXFP4
# experts, bf16 attention, router and head
C3 = Config("c3-gptoss-moe", 24, 2880, 2880, 64, 8, 64, 201088, A.HC_FMT_MXFP4, norm_scale=False,
            rope_theta=150000.0, norm_eps=1e-5, arch="gptoss", experts=32, top_k=4, window=128,
            attn_fmt=A.HC_FMT_BF16, yarn=(32.0, 32.0, 1.0, 4096, False))
CONFIGS = {"c1": C1, "c2": C2, "c3": C3, "c4_draft": C4_DRAFT}


def bf16_bits(x):
    """float32 -> bf16 bits, round to nearest even (NaN-free inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _ptr(a):
    return C.c_void_p(a.ctypes.data) if a is not None else C.c_void_p()


def _f32(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def normal(seed, name, n, std):
    out = np.empty(n, dtype=np.float32)
    sd = np.array([std], np.float32)
    A.check(A.lib().hc_synth_normal(seed, name.encode(), _f32(sd), _f32(out), n))
    return out


def tokens(seed, vocab, n):
    out = np.empty(n, dtype=np.int32)
    A.check(A.lib().hc_synth_tokens(seed, vocab, out.ctypes.data_as(C.POINTER(C.c_int32)), n))
    return out


def f16_bits(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    A.lib().hc_f32_to_f16(_f32(x), out.ctypes.data_as(C.POINTER(C.c_uint16)), x.size)
    return out


def f16_values(h):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    A.lib().hc_f16_to_f32(h.ctypes.data_as(C.POINTER(C.c_uint16)), _f32(out), h.size)
    return out


class Linear:
    """One matrix in a reference byte layout (the arrays hc_linear_desc points to)."""

    def __init__(self, fmt, rows, cols, data, scales=None, zeros=None, exps=None, bias=None):
        self.fmt, self.rows, self.cols = fmt, rows, cols
        self.data, self.scales, self.zeros, self.exps, self.bias = data, scales, zeros, exps, bias

    def desc(self):
        bias = None if self.bias is None else np.ascontiguousarray(self.bias, np.float32)
        self.bias = bias
        return A.LinearDesc(self.fmt, self.rows, self.cols, _ptr(self.data), _ptr(self.scales),
                            _ptr(self.zeros), _ptr(self.exps), _ptr(bias))

    @staticmethod
    def quantize(w, fmt, search=False):
        """palette.QuantizeLinear (int8 a scale a row; int4 symmetric, 32 a scale), the
        asymmetric int4 quantiser, or mxfp4.Encode, through the library's converter."""
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        L = A.lib()
        u8 = C.POINTER(C.c_uint8)
        u16 = C.POINTER(C.c_uint16)
        if fmt == A.HC_FMT_INT8_ROW:
            data = np.empty(rows * cols, np.uint8)
            sc = np.empty(rows, np.uint16)
            A.check(L.hc_quantize_linear(_f32(w), rows, cols, 0, 8, int(search), data.ctypes.data_as(u8), sc.ctypes.data_as(u16)))
            return Linear(fmt, rows, cols, data, scales=sc)
        if fmt == A.HC_FMT_INT4_SYM_G32:
            data = np.empty(rows * cols // 2, np.uint8)
            sc = np.empty(rows * cols // 32, np.uint16)
            A.check(L.hc_quantize_linear(_f32(w), rows, cols, 32, 4, int(search), data.ctypes.data_as(u8), sc.ctypes.data_as(u16)))
            return Linear(fmt, rows, cols, data, scales=sc)
        if fmt == A.HC_FMT_INT4_ASYM_G32:
            data = np.empty(rows * cols // 2, np.uint8)
            sc = np.empty(rows * cols // 32, np.uint16)
            z = np.empty(rows * cols // 32, np.uint16)
            A.check(L.hc_quantize_int4_asym(_f32(w), rows, cols, data.ctypes.data_as(u8), sc.ctypes.data_as(u16), z.ctypes.data_as(u16)))
            return Linear(fmt, rows, cols, data, scales=sc, zeros=z)
        if fmt == A.HC_FMT_MXFP4:
            data = np.empty(rows * cols // 2, np.uint8)
            e = np.empty(rows * cols // 32, np.uint8)
            A.check(L.hc_mxfp4_encode(_f32(w), rows, cols, data.ctypes.data_as(u8), e.ctypes.data_as(u8)))
            return Linear(fmt, rows, cols, data, exps=e)
        raise ValueError(f"format {fmt}")


class LibGen:
    """The synthetic-weight generator and quantisers of libhwnpu_cuda.so."""

    normal = staticmethod(normal)
    tokens = staticmethod(tokens)
    f16_bits = staticmethod(f16_bits)

    @staticmethod
    def quantize(w, fmt, search=False):
        return Linear.quantize(w, fmt, search)


class Model:
    """A synthetic model of a Config: quantised weights plus norms, and its hc_model_desc."""

    def __init__(self, cfg: Config, seed: int = 0, norm_std: float = 0.0, gen=LibGen):
        self.cfg = cfg
        c = cfg
        hd = c.head_dim
        if c.arch == "gptoss":
            self._gptoss(gen, seed, norm_std)
            return

        def mat(name, rows, cols):
            w = gen.normal(seed, name, rows * cols, c.std).reshape(rows, cols)
            return gen.quantize(w, c.fmt, c.quant_search)

        def norm(name, n):
            if norm_std == 0.0:
                return gen.f16_bits(np.ones(n, np.float32))
            return gen.f16_bits(1.0 + gen.normal(seed, name, n, norm_std))

        self.layers = []
        for i in range(c.layers):
            p = f"model.layers.{i}."
            L = {
                "input_norm": norm(p + "input_layernorm.weight", c.hidden),
                "post_norm": norm(p + "post_attention_layernorm.weight", c.hidden),
                "q": mat(p + "self_attn.q_proj.weight", c.heads * hd, c.hidden),
                "k": mat(p + "self_attn.k_proj.weight", c.kv_heads * hd, c.hidden),
                "v": mat(p + "self_attn.v_proj.weight", c.kv_heads * hd, c.hidden),
                "o": mat(p + "self_attn.o_proj.weight", c.hidden, c.heads * hd),
                "gate": mat(p + "mlp.gate_proj.weight", c.inter, c.hidden),
                "up": mat(p + "mlp.up_proj.weight", c.inter, c.hidden),
                "down": mat(p + "mlp.down_proj.weight", c.hidden, c.inter),
            }
            if c.qk_norm:
                L["q_norm"] = norm(p + "self_attn.q_norm.weight", hd)
                L["k_norm"] = norm(p + "self_attn.k_norm.weight", hd)
            self.layers.append(L)
        self.final_norm = norm("model.norm.weight", c.hidden)
        if c.tied:
            self.head = mat("model.embed_tokens.weight", c.vocab, c.hidden)
            self.embed = None
        else:
            self.head = mat("lm_head.weight", c.vocab, c.hidden)
            self.embed = gen.f16_bits(gen.normal(seed, "model.embed_tokens.weight", c.vocab * c.hidden, c.std))
        self._desc = None

    def _gptoss(self, gen, seed, norm_std):
        """gpt-oss's tensors (gptoss/config.go HostExperts, build.go): bf16 q/k/v/o with float32
        biases, sinks N(0, 1), a router drawn N(0, 1 / hidden) so that its logits are about N(0, 1)
        MXFP4 experts (mxfp4.Encode of N(0, std^2)) with biases, an untied
        bf16 head and an fp16 embedding."""
        c = self.cfg
        hd, E, I, D = c.head_dim, c.experts, c.inter, c.hidden
        af = c.attn_fmt if c.attn_fmt >= 0 else c.fmt

        def mat(name, rows, cols, std=c.std, fmt=af):
            w = gen.normal(seed, name, rows * cols, std).reshape(rows, cols)
            if fmt == A.HC_FMT_BF16:
                return Linear(fmt, rows, cols, bf16_bits(w))
            return gen.quantize(w, fmt, c.quant_search)

        def vec(name, n, std):
            return gen.normal(seed, name, n, std)

        def norm(name, n):
            if norm_std == 0.0:
                return gen.f16_bits(np.ones(n, np.float32))
            return gen.f16_bits(1.0 + gen.normal(seed, name, n, norm_std))

        self.layers = []
        for i in range(c.layers):
            p = f"model.layers.{i}."
            L = {"input_norm": norm(p + "input_layernorm.weight", D),
                 "post_norm": norm(p + "post_attention_layernorm.weight", D)}
            for k, rows, cols in (("q", c.heads * hd, D), ("k", c.kv_heads * hd, D), ("v", c.kv_heads * hd, D),
                                  ("o", D, c.heads * hd)):
                L[k] = mat(p + f"self_attn.{k}_proj.weight", rows, cols)
                L[k].bias = vec(p + f"self_attn.{k}_proj.bias", rows, c.std)
            L["sinks"] = vec(p + "self_attn.sinks", c.heads, 1.0)
            L["window"] = c.window if i % 2 == 0 else 0
            L["router"] = mat(p + "mlp.router.weight", E, D, std=1.0 / np.sqrt(D))
            L["router"].bias = vec(p + "mlp.router.bias", E, c.std)
            L["experts_gate_up"] = mat(p + "mlp.experts.gate_up_proj", E * 2 * I, D, fmt=A.HC_FMT_MXFP4)
            L["experts_gate_up"].bias = vec(p + "mlp.experts.gate_up_proj_bias", E * 2 * I, c.std)
            L["experts_down"] = mat(p + "mlp.experts.down_proj", E * D, I, fmt=A.HC_FMT_MXFP4)
            L["experts_down"].bias = vec(p + "mlp.experts.down_proj_bias", E * D, c.std)
            self.layers.append(L)
        self.final_norm = norm("model.norm.weight", D)
        self.head = mat("lm_head.weight", c.vocab, D)
        self.embed = gen.f16_bits(gen.normal(seed, "model.embed_tokens.weight", c.vocab * D, c.std))
        self._desc = None

    def desc(self):
        c = self.cfg
        layers = (A.LayerDesc * c.layers)()
        none = A.LinearDesc(A.HC_FMT_NONE, 0, 0, None, None, None, None, None)
        for i, L in enumerate(self.layers):
            d = layers[i]
            d.input_norm, d.post_norm = _ptr(L["input_norm"]), _ptr(L["post_norm"])
            d.q_norm, d.k_norm = _ptr(L.get("q_norm")), _ptr(L.get("k_norm"))
            for k in ("q", "k", "v", "o", "gate", "up", "down", "router", "experts_gate_up", "experts_down"):
                setattr(d, k, L[k].desc() if k in L else none)
            d.sinks = _ptr(L.get("sinks"))
            d.sliding_window = L.get("window", 0)
        gpt = c.arch == "gptoss"
        flags = (A.HC_MODEL_QK_NORM if c.qk_norm else 0) | (A.HC_MODEL_TIED if c.tied else 0) | \
                (A.HC_MODEL_NORM_SCALE if c.norm_scale else 0) | (A.HC_MODEL_ATTN_BIAS if gpt else 0)
        md = A.ModelDesc()
        md.abi, md.arch, md.flags = A.HC_ABI, A.HC_ARCH_GPTOSS if gpt else A.HC_ARCH_QWEN3, flags
        md.hidden, md.inter, md.layers = c.hidden, c.inter, c.layers
        md.heads, md.kv_heads, md.head_dim, md.vocab = c.heads, c.kv_heads, c.head_dim, c.vocab
        md.experts, md.top_k = c.experts, c.top_k
        md.norm_eps, md.rope_theta = c.norm_eps, c.rope_theta
        md.yarn_factor, md.yarn_beta_fast, md.yarn_beta_slow = (c.yarn[0], c.yarn[1], c.yarn[2]) if gpt else (1.0, 0.0, 0.0)
        md.yarn_original, md.yarn_truncate = (c.yarn[3], int(c.yarn[4])) if gpt else (0, 0)
        md.swiglu_alpha, md.swiglu_limit = c.swiglu
        md.embed = _ptr(self.embed)
        md.final_norm = _ptr(self.final_norm)
        md.head = self.head.desc()
        md.layer = C.cast(layers, C.POINTER(A.LayerDesc))
        self._desc = (md, layers)  # keep the layer array alive with the descriptor
        return md

    def weight_bytes(self):
        """Bytes of the model's weights in their reference layouts."""
        n = 0
        for L in self.layers:
            for k, v in L.items():
                if isinstance(v, Linear) and not k.startswith("experts"):
                    n += sum(a.nbytes for a in (v.data, v.scales, v.zeros, v.exps) if a is not None)
        h = self.head
        n += sum(a.nbytes for a in (h.data, h.scales, h.zeros, h.exps) if a is not None)
        return n
