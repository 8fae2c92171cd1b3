"""The CPU oracle pinned against the reference's own known-answer tests (ported; the Go
reference cannot run here) and against an independent float64 forward. No GPU."""

import ctypes as C
from dataclasses import replace
import math

import numpy as np
import pytest

import oracle_lib as O
from hwnpu_b200 import _abi as A
from hwnpu_b200 import synth

L = O.lib


def f16(x):
    return L().or_f16_bits(float(x))


def test_f16_all_halves_round_trip():
    # vecops TestF16 (internal/vecops/vecops_test.go:421-486): every half that is not a NaN
    # comes back bit for bit; NaNs become sign|0x7e00
    for h in range(1 << 16):
        v = L().or_f16_value(h)
        if (h & 0x7C00) == 0x7C00 and (h & 0x3FF):
            assert L().or_f16_bits(v) == (h & 0x8000) | 0x7E00
            continue
        assert L().or_f16_bits(v) == h, hex(h)
        assert np.float16(v).view(np.uint16) == h


def test_f16_rne_matches_numpy_and_product():
    rng = np.random.default_rng(5)
    bits = rng.integers(0, 1 << 32, 20000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = np.where(np.isnan(x), np.float32(1.0), x)
    want = x.astype(np.float16).view(np.uint16)
    got = np.array([L().or_f16_bits(float(v)) for v in x[:4000]], np.uint16)
    assert np.array_equal(got, want[:4000])
    assert np.array_equal(synth.f16_bits(x), want)  # the product's converter


def test_exp_cephes():
    # f32.Exp is within 2 ulp (internal/f32/f32.go:6-9)
    for v in np.linspace(-80, 80, 2001, dtype=np.float32):
        got = L().or_exp(float(v))
        want = math.exp(float(v))
        assert abs(got - want) <= 3 * np.spacing(np.float32(want)), v


def test_constexpr_int4_known_answer():
    # milcpu TestConstexpr (internal/milcpu/milcpu_test.go:297-309): data 0x21 0xF0 0x87 0x00 with
    # scales 0.5 and 2 is rows [1 2 0 -1]*0.5 and [7 -8 0 0]*2
    data = np.array([0x21, 0xF0, 0x87, 0x00], np.uint8)
    sc = np.array([f16(0.5), f16(2)], np.uint16)
    out = np.empty(8, np.float32)
    L().or_dequant_linear(O.p(data, O._u8p), O.p(sc, O._u16p), 2, 4, 4, 4, O.p(out, O._f32p))
    assert out.reshape(2, 4).T.ravel().tolist() == [0.5, 14, 1, -16, 0, 0, -0.5, 0]


def quantize_both(w, rows, cols, block, bits, search):
    n = rows * cols if bits == 8 else rows * cols // 2
    nb = rows * (cols // (block or cols))
    d1, s1 = np.zeros(n, np.uint8), np.zeros(nb, np.uint16)
    L().or_quantize_linear(O.p(w, O._f32p), rows, cols, block, bits, int(search), O.p(d1, O._u8p), O.p(s1, O._u16p))
    d2, s2 = np.zeros(n, np.uint8), np.zeros(nb, np.uint16)
    A.check(A.lib().hc_quantize_linear(O.p(w, O._f32p), rows, cols, block, bits, int(search),
                                       O.p(d2, O._u8p), O.p(s2, O._u16p)))
    assert np.array_equal(d1, d2) and np.array_equal(s1, s2), "product quantiser differs from the oracle"
    out = np.empty(rows * cols, np.float32)
    L().or_dequant_linear(O.p(d1, O._u8p), O.p(s1, O._u16p), rows, cols, block or cols, bits, O.p(out, O._f32p))
    return out


@pytest.mark.parametrize("bits,block,search,bound", [(8, 0, False, 0.01), (4, 0, False, 0.15), (4, 0, True, 0.12),
                                                     (4, 128, False, 0.125), (4, 128, True, 0.11), (4, 32, False, 0.11)])
def test_quantize_linear_error_bounds(bits, block, search, bound):
    # palette TestQuantizeLinear (internal/palette/palette_test.go:110-133); 33 rows, N(0, 1)
    w = np.random.default_rng(1).standard_normal(33 * 1024).astype(np.float32)
    back = quantize_both(w, 33, 1024, block, bits, search)
    e = math.sqrt(float(((w - back) ** 2).sum() / (w ** 2).sum()))
    assert e < bound


def test_quantize_linear_exact_levels():
    # palette_test.go:133-141: exact levels come back exactly
    w = np.array([-7, -1, 0, 3, 7, 2], np.float32)
    assert quantize_both(w, 1, 6, 0, 4, False).tolist() == [-7, -1, 0, 3, 7, 2]


def test_int4_asym_quantiser_product_equals_oracle():
    rng = np.random.default_rng(2)
    rows, cols = 17, 512
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    w[:32] = 0.25          # a constant block
    w[32:64] = 0.0         # a block of zeros
    outs = []
    for fn in (lambda *a: L().or_quantize_int4_asym(*a), lambda *a: A.check(A.lib().hc_quantize_int4_asym(*a))):
        d, s, z = np.zeros(rows * cols // 2, np.uint8), np.zeros(rows * cols // 32, np.uint16), np.zeros(rows * cols // 32, np.uint16)
        fn(O.p(w, O._f32p), rows, cols, O.p(d, O._u8p), O.p(s, O._u16p), O.p(z, O._u16p))
        outs.append((d, s, z))
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    d, s, z = outs[0]
    back = np.empty(rows * cols, np.float32)
    L().or_dequant_int4_asym(O.p(d, O._u8p), O.p(s, O._u16p), O.p(z, O._u16p), rows, cols, O.p(back, O._f32p))
    assert np.all(back[:32] == 0.25) and np.all(back[32:64] == 0)
    # within half a step (plus fp16 rounding of s and z) of every value
    step = synth.f16_values(s).repeat(32)
    assert np.all(np.abs(back - w) <= step * 0.5 + step * 16 * 2 ** -10 + 1e-9)
    assert math.sqrt(((w - back) ** 2).sum() / (w ** 2).sum()) < 0.1


def test_mxfp4_nearest_table():
    # mxfp4 TestEncode's nearest() cases (internal/mxfp4/mxfp4_test.go:168-175)
    cases = [(0.25, 0), (0.26, 1), (0.75, 2), (1.25, 2), (1.75, 4), (2.5, 4), (3.5, 6), (5, 6), (5.1, 7),
             (100, 7), (-0.6, 9), (-0.1, 0)]
    for x, want in cases:
        assert L().or_mxfp4_nearest(x) == want, x


def mx_encode_both(row):
    n = row.size
    outs = []
    for fn in (lambda r, w, e: L().or_mxfp4_encode(O.p(r, O._f32p), n, O.p(w, O._u8p), O.p(e, O._u8p)),
               lambda r, w, e: A.check(A.lib().hc_mxfp4_encode(O.p(r, O._f32p), 1, n, O.p(w, O._u8p), O.p(e, O._u8p)))):
        w, e = np.zeros(n // 2, np.uint8), np.zeros(n // 32, np.uint8)
        fn(row, w, e)
        outs.append((w, e))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    return outs[0]


def test_mxfp4_encode_properties():
    # mxfp4 TestEncode (internal/mxfp4/mxfp4_test.go:120-166)
    rng = np.random.default_rng(3)
    nb = 64
    row = (rng.standard_normal(nb * 32) * 0.02).astype(np.float32)
    row[5] = 0
    row[32:64] = 0
    w, e = mx_encode_both(row)
    got = np.empty(row.size, np.float32)
    L().or_mxfp4_dequant(O.p(w, O._u8p), O.p(e, O._u8p), row.size, O.p(got, O._f32p))
    assert got[5] == 0 and got[32] == 0
    for b in range(nb):
        s = 2.0 ** (int(e[b]) - 127)
        for j in range(32):
            v, d = row[b * 32 + j], row[b * 32 + j] - got[b * 32 + j]
            if v != 0 and abs(v) / s < 6:
                assert abs(d) <= s + 1e-12
    rel = math.sqrt(float(((row - got) ** 2).sum() / (row ** 2).sum()))
    assert rel < 0.12


def test_mxfp4_dot_matches_dequantized_product():
    # mxfp4 TestDot (internal/mxfp4/mxfp4_test.go:21-55)
    rng = np.random.default_rng(12)
    for nb in (1, 2, 3, 90):
        w = rng.integers(0, 256, 16 * nb, dtype=np.uint8)
        e = rng.integers(118, 126, nb, dtype=np.uint8)
        x = rng.standard_normal(nb * 32).astype(np.float32)
        q, s = np.empty(nb * 32, np.int8), np.empty(nb, np.float32)
        L().or_mxfp4_quantize(O.p(x, O._f32p), nb * 32, O.p(q, O._i8p), O.p(s, O._f32p))
        row = np.empty(nb * 32, np.float32)
        L().or_mxfp4_dequant(O.p(w, O._u8p), O.p(e, O._u8p), nb * 32, O.p(row, O._f32p))
        want = 0.0
        for b in range(nb):
            for j in range(16):
                want += float(row[b * 32 + 2 * j]) * float(q[b * 32 + j]) * float(s[b])
                want += float(row[b * 32 + 2 * j + 1]) * float(q[b * 32 + 16 + j]) * float(s[b])
        got = L().or_mxfp4_dot(O.p(w, O._u8p), O.p(e, O._u8p), nb * 32, O.p(q, O._i8p), O.p(s, O._f32p))
        assert abs(got - want) <= 1e-4 * max(1, abs(want))
        exact = float(np.dot(row.astype(np.float64), x.astype(np.float64)))
        assert abs(want - exact) <= 0.01 * math.sqrt(float((row.astype(np.float64) ** 2).sum() * (x.astype(np.float64) ** 2).sum()))


def merge(parts, sinks=None, tokens=1):
    rows, dim = parts[0][0].shape
    m = L().or_merge_new(rows, dim)
    for o, mx, l in parts:
        L().or_merge_add(m, O.p(np.ascontiguousarray(o, np.float32), O._f32p), O.p(np.ascontiguousarray(mx, np.float32), O._f32p),
                         O.p(np.ascontiguousarray(l, np.float32), O._f32p))
    if sinks is not None:
        L().or_merge_add_sink(m, O.p(np.asarray(sinks, np.float32), O._f32p), tokens)
    out = np.empty((rows, dim), np.float32)
    L().or_merge_result(m, O.p(out, O._f32p))
    L().or_merge_free(m)
    return out


def test_merge_order():
    # paged TestMergeOrder (internal/llm/paged/paged_test.go:133-156)
    o = [np.array([[1, 2]]), np.array([[3, 4]]), np.array([[5, 6]])]
    m = [[-1], [4], [2]]
    l = [[2], [1], [3]]
    w = sum(l[j][0] * math.exp(m[j][0] - 4) for j in range(3))
    x0 = sum(l[j][0] * math.exp(m[j][0] - 4) * o[j][0][0] for j in range(3)) / w
    x1 = sum(l[j][0] * math.exp(m[j][0] - 4) * o[j][0][1] for j in range(3)) / w
    for order in ([0, 1, 2], [2, 1, 0], [1, 0, 2]):
        out = merge([(o[j], m[j], l[j]) for j in order])
        assert abs(out[0][0] - x0) <= 1e-5 and abs(out[0][1] - x1) <= 1e-5


def test_merge_sink():
    # paged TestMergeSink (internal/llm/paged/paged_test.go:160-186)
    scores, vals, sink = [0.5, -1, 2], [[1, 2], [3, -1], [0.5, 4]], 1.5
    tot = sum(math.exp(s) for s in scores) + math.exp(sink)
    want = [sum(math.exp(s) / tot * vals[i][j] for i, s in enumerate(scores)) for j in range(2)]
    out = merge([(np.array([vals[i]]), [s], [1]) for i, s in enumerate(scores)], sinks=[sink])
    assert np.allclose(out[0], want, atol=1e-5)


def test_merge_matches_full_softmax():
    # paged TestMergeMatchesFull (paged_test.go:17-131): chunks of a cache merged equal one softmax
    rng = np.random.default_rng(4)
    d, chunk, chunks = 16, 16, 4
    q = rng.standard_normal(d)
    k = rng.standard_normal((chunk * chunks, d))
    v = rng.standard_normal((chunk * chunks, d))
    s = k @ q / math.sqrt(d)
    p = np.exp(s - s.max())
    want = (p / p.sum()) @ v
    parts = []
    for c in range(chunks):
        sc = s[c * chunk:(c + 1) * chunk]
        mx = sc.max()
        pe = np.exp(sc - mx)
        parts.append((np.array([(pe / pe.sum()) @ v[c * chunk:(c + 1) * chunk]]), [mx], [pe.sum()]))
    assert np.allclose(merge(parts)[0], want, atol=1e-5)


def test_route_softmax_topk_stable():
    # experts.Routing.Choose (experts/weights.go:33-82): softmax, stable descending, top k, renorm
    logits = np.array([1.0, 3.0, 3.0, -2.0, 0.5, 3.0], np.float32)
    idx, w = np.zeros(4, np.int32), np.zeros(4, np.float32)
    L().or_route(O.p(logits, O._f32p), 6, 4, 1, O.p(idx, O._i32p), O.p(w, O._f32p))
    assert idx.tolist() == [1, 2, 5, 0]  # ties keep the lower expert first
    sm = np.exp(logits - logits.max()) / np.exp(logits - logits.max()).sum()
    ww = sm[[1, 2, 5, 0]] / (sm[[1, 2, 5, 0]].sum() + 1e-6)
    assert np.allclose(w, ww, rtol=1e-6)


def test_argmax_first_of_equal():
    # chat.Sampling.pick at temperature 0 keeps the first of equal maxima (sample.go:80-88)
    v = np.array([0.5, 2.0, -1.0, 2.0], np.float32)
    assert L().or_argmax(O.p(v, O._f32p), 4) == 1
    h = synth.f16_bits(v)
    assert L().or_argmax_f16(O.p(h, O._u16p), 4) == 1


TINY = synth.Config("tiny-qwen3", 2, 256, 512, 4, 2, 64, 1000, A.HC_FMT_INT4_ASYM_G32, tied=True, qk_norm=True,
                    rope_theta=1e6, std=0.05)
TINY_LLAMA = synth.Config("tiny-llama", 2, 256, 768, 8, 2, 32 * 2, 1200, A.HC_FMT_INT8_ROW, std=0.05)


def rel(a, b):
    return float(np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum()))


@pytest.mark.parametrize("cfg", [TINY, TINY_LLAMA], ids=lambda c: c.name)
def test_oracle_matches_float64_forward(cfg):
    # qwen3 TestMatchesReference (internal/llm/qwen3/qwen3_test.go:297-350): the CPU interpreter's
    # logits against a float64 forward written from the model definition
    import ref_f64

    model = synth.Model(cfg, seed=11, norm_std=0.1)
    toks = synth.tokens(5, cfg.vocab, 9)
    want = ref_f64.forward(model, toks)
    s = O.OracleSession(model, 32)
    got = synth.f16_values(s.step(toks, all_rows=True)).astype(np.float64)
    s.close()
    # fp16 logits, fp16 RoPE tables and scale constants: a few 1e-4
    assert rel(got, want) < 2e-3, rel(got, want)


@pytest.mark.parametrize("q", [1, 3, 4])
def test_oracle_cached_matches_full(q):
    # qwen3 TestCachedMatchesFull (internal/llm/qwen3/cache_test.go:187-213): stepping with the
    # fp16 KV cache against one pass over all tokens, worst relative error <= 5e-3
    model = synth.Model(TINY, seed=13, norm_std=0.1)
    toks = synth.tokens(6, TINY.vocab, 11)
    full = O.OracleSession(model, 32)
    ref = synth.f16_values(full.step(toks, all_rows=True))
    s = O.OracleSession(model, 32)
    worst, pos = 0.0, 0
    while pos < len(toks):
        v = min(q, len(toks) - pos)
        got = synth.f16_values(s.step(toks[pos:pos + v])[0])
        pos += v
        worst = max(worst, rel(got, ref[pos - 1]))
    full.close()
    s.close()
    assert worst <= 5e-3


def test_oracle_speculate_equals_plain():
    # chat TestSpeculate (internal/chat/engine_test.go:348-478): speculative greedy output is the
    # plain greedy output
    model = synth.Model(TINY, seed=17, norm_std=0.1)
    prompt = list(synth.tokens(7, TINY.vocab, 6))
    plain = O.OracleSession(model, 64)
    out_plain = []
    logits = plain.step(prompt)[0]
    for _ in range(12):
        t = L().or_argmax_f16(O.p(logits, O._u16p), TINY.vocab)
        out_plain.append(t)
        logits = plain.step([t])[0]
    spec = O.OracleSession(model, 64)
    first = spec.step(prompt)[0]
    nxt = L().or_argmax_f16(O.p(first, O._u16p), TINY.vocab)
    out = [nxt]
    rng = np.random.default_rng(1)
    while len(out) < 12:
        # drafts: the plain output where known, a wrong token now and then
        k = len(out)
        drafts = [out_plain[k + i] if k + i < len(out_plain) and rng.random() > 0.3 else int(rng.integers(TINY.vocab)) for i in range(3)]
        kept, nxt, _ = spec.speculate([out[-1]] + drafts)
        out.extend(drafts[:kept - 1])
        out.append(nxt)
    assert out[:12] == out_plain
    plain.close()
    spec.close()


def test_oracle_paged_int8_close_to_fp16():
    # the oracle's restatement of the paged int8 cache (this library's own format; no reference):
    # stepping token by token across page boundaries (scales grow, earlier rows get requantised)
    # stays close to the fp16 cache
    model = synth.Model(TINY, seed=19, norm_std=0.1)
    toks = list(synth.tokens(8, TINY.vocab, 40))
    f16 = O.OracleSession(model, 64)
    pg = O.OracleSession(model, 64, kv_format=A.HC_KV_INT8_PAGED, share=f16)
    f16.step(toks[:5])
    pg.step(toks[:5])
    for t in toks[5:]:
        a = synth.f16_values(f16.step([t])[0])
        b = synth.f16_values(pg.step([t])[0])
        assert np.abs(a - b).max() <= 5e-2 * np.abs(a).max()
    pg.close()
    f16.close()


def _page_write_np(rows, scale_bits, off, x):
    """The paged int8 cache's write rule restated in numpy float32: the page scale is the fp16
    rounding up of max|x| / 127 over its rows; a row that needs a larger scale requantises the
    earlier rows to it (q' = round_even(q * (s_old / s_new)), clamped to +-127); the row is then
    round_even(x * (1 / s)), clamped."""
    f32 = np.float32
    m = f32(np.abs(x).max())
    s_old = f32(0) if off == 0 else f32(np.uint16(scale_bits).view(np.float16))
    s_new = s_old
    need = f32(m / f32(127))
    if need > s_old:
        h = np.float16(need)
        if f32(h) < need:
            h = np.nextafter(h, np.float16(np.inf))
        s_new = f32(h)
        if off > 0 and s_old > 0:
            fac = f32(s_old / s_new)
            rows[:off] = np.clip(np.rint(rows[:off].astype(f32) * fac), -127, 127).astype(np.int8)
        scale_bits = int(np.float16(s_new).view(np.uint16))
    inv = f32(f32(1) / s_new) if s_new > 0 else f32(0)
    rows[off] = np.clip(np.rint(x.astype(f32) * inv), -127, 127).astype(np.int8)
    return scale_bits


def test_oracle_page_write_matches_restatement():
    # the oracle's page writes (or_page_write, the rule its int8-paged sessions use) against an
    # independent numpy restatement, byte for byte, over pages whose rows grow, shrink and jump in
    # magnitude (so scales grow and earlier rows are requantised, several times a page)
    rng = np.random.default_rng(5)
    hd = 128
    for page in range(40):
        got = np.zeros((16, hd), np.int8)
        want = np.zeros((16, hd), np.int8)
        gs = C.c_uint16(0)
        ws = 0
        for off in range(16):
            x = (rng.standard_normal(hd) * rng.choice([0.01, 0.1, 1.0, 7.0, 40.0])).astype(np.float32)
            if page % 7 == 0 and off == 3:
                x[:] = 0.0  # an all-zero row keeps the scale
            L().or_page_write(O.p(got, O._i8p), C.byref(gs), off, O.p(x, O._f32p), hd)
            ws = _page_write_np(want, ws, off, x)
            assert int(gs.value) == ws, (page, off)
            assert np.array_equal(got, want), (page, off)


# a gpt-oss-shaped model small enough for the CPU: sliding layers of a window of 8 alternate with
# full ones, 8 experts, top 2
TINY_GPTOSS = synth.Config("tiny-gptoss", 2, 256, 256, 4, 2, 64, 500, A.HC_FMT_MXFP4, norm_scale=False,
                           rope_theta=150000.0, norm_eps=1e-5, arch="gptoss", experts=8, top_k=2, window=8,
                           attn_fmt=A.HC_FMT_BF16, yarn=(32.0, 32.0, 1.0, 4096, False))


def test_oracle_yarn_matches_formula():
    # gptoss.Config.RopeInvFreq (gptoss/config.go:136-166) restated in numpy: the oracle's rotary
    # tables (scaled by 0.1 ln(factor) + 1) drive its logits; a model with YaRN off differs
    dim, theta, factor, bf, bs, orig = 64, 150000.0, 32.0, 32.0, 1.0, 4096
    corr = lambda rot: dim * np.log(orig / (rot * 2 * np.pi)) / (2 * np.log(theta))
    low, high = max(corr(bf), 0.0), min(corr(bs), dim - 1.0)
    i = np.arange(dim // 2)
    pos = theta ** (2 * i / dim)
    ramp = np.clip((i - low) / (high - low), 0, 1)
    inv = (1 / (factor * pos)) * ramp + (1 / pos) * (1 - ramp)
    assert inv[0] == 1.0 and abs(inv[-1] - 1 / (factor * pos[-1])) < 1e-15
    model = synth.Model(TINY_GPTOSS, seed=3, norm_std=0.1)
    plain = synth.Model(replace(TINY_GPTOSS, yarn=(1.0, 32.0, 1.0, 4096, False)), seed=3, norm_std=0.1)
    toks = list(synth.tokens(4, TINY_GPTOSS.vocab, 12))
    a, b = O.OracleSession(model, 32), O.OracleSession(plain, 32)
    la, lb = a.step(toks)[0], b.step(toks)[0]
    assert not np.array_equal(la, lb)
    a.close()
    b.close()


def test_oracle_gptoss_cached_matches_full():
    # TestCachedMatchesFull's property for gpt-oss: stepping token by token over the caches (a
    # sliding window of 8 crossed) equals one pass. The bound is twice qwen3's 5e-3: the fp16 cache
    # against the pass's float32 keys moves moe_x a little, and its int8 quantisation per 32 in the
    # experts (mxfp4.Vec.Quantize) turns that into whole steps of 1/127 of a group's largest value
    model = synth.Model(TINY_GPTOSS, seed=5, norm_std=0.1)
    toks = synth.tokens(6, TINY_GPTOSS.vocab, 14)
    full = O.OracleSession(model, 32)
    ref = synth.f16_values(full.step(toks, all_rows=True))
    s = O.OracleSession(model, 32, share=full)
    worst = 0.0
    for i, t in enumerate(toks):
        got = synth.f16_values(s.step([t])[0])
        worst = max(worst, rel(got, ref[i]))
    s.close()
    full.close()
    assert worst <= 1e-2, worst
