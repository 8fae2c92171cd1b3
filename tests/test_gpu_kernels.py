"""Kernel parity on a B200 through the C ABI: bit-exact dequantisation of every format, the
decode GEMV, split-K attention, greedy choice and MoE routing against the CPU oracle or a
float64 reference."""

import ctypes as C

import numpy as np
import pytest

import hwnpu_b200 as hb
import oracle_lib as O
from hwnpu_b200 import _abi as A
from hwnpu_b200 import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def oracle_dequant(lin):
    import ref_f64

    return ref_f64.dequant(lin).astype(np.float32)


class Loaded:
    def __init__(self, device, lin):
        self.lin = lin
        h = C.c_void_p()
        A.check(A.lib().hc_linear_load(device.h, C.byref(lin.desc()), C.byref(h)))
        self.h = h

    def dequant(self):
        out = np.empty((self.lin.rows, self.lin.cols), np.float32)
        A.check(A.lib().hc_linear_dequant(self.h, 0, self.lin.rows, out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def run(self, x):
        xt = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        yt = torch.empty((x.shape[0], self.lin.rows), dtype=torch.float32, device="cuda")
        A.check(A.lib().hc_linear_run(self.h, C.c_void_p(xt.data_ptr()), x.shape[0], C.c_void_p(yt.data_ptr()), None))
        torch.cuda.synchronize()
        return yt.cpu().numpy()

    def close(self):
        A.lib().hc_linear_free(self.h)


FORMATS = [A.HC_FMT_INT8_ROW, A.HC_FMT_INT4_SYM_G32, A.HC_FMT_INT4_ASYM_G32, A.HC_FMT_MXFP4]
SHAPES = [(40, 2048), (100, 2816 // 32 * 32), (37, 6144), (256, 1024), (64, 2880), (8, 64), (4104, 768)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_dequant_bit_exact(device, fmt, shape):
    rows, cols = shape
    w = synth.normal(3, f"w{rows}x{cols}", rows * cols, 0.02).reshape(rows, cols)
    lin = synth.Linear.quantize(w, fmt)
    d = Loaded(device, lin)
    got = d.dequant()
    d.close()
    want = oracle_dequant(lin)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_int4_known_answer_through_tiles(device):
    # milcpu TestConstexpr's int4 rows (milcpu_test.go:297-309) inside a 2 x 32 matrix
    data = np.zeros(32, np.uint8)
    data[:2] = [0x21, 0xF0]        # row 0: 1 2 0 -1
    data[16:18] = [0x87, 0x00]     # row 1: 7 -8 0 0
    sc = synth.f16_bits(np.array([0.5, 2], np.float32))
    lin = synth.Linear(A.HC_FMT_INT4_SYM_G32, 2, 32, data, scales=sc)
    d = Loaded(device, lin)
    got = d.dequant()
    d.close()
    assert got[0, :4].tolist() == [0.5, 1, 0, -0.5] and got[1, :4].tolist() == [14, -16, 0, 0]
    assert not got[:, 4:].any()


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("ntok", [1, 3, 8, 11, 37, 64, 70])
def test_gemv(device, fmt, shape, ntok):
    rows, cols = shape
    w = synth.normal(5, f"g{rows}x{cols}", rows * cols, 0.02).reshape(rows, cols)
    lin = synth.Linear.quantize(w, fmt)
    x = synth.normal(6, f"x{ntok}", ntok * cols, 1.0).reshape(ntok, cols)
    d = Loaded(device, lin)
    got = d.run(x)
    d.close()
    if fmt == A.HC_FMT_MXFP4:
        # the reference's own arithmetic: int8 vector blocks, integer block sums (mxfp4.go:33-91)
        want = np.empty((ntok, rows), np.float32)
        for t in range(ntok):
            q, s = np.empty(cols, np.int8), np.empty(cols // 32, np.float32)
            xt = np.ascontiguousarray(x[t])
            O.lib().or_mxfp4_quantize(O.p(xt, O._f32p), cols, O.p(q, O._i8p), O.p(s, O._f32p))
            for r in range(rows):
                want[t, r] = O.lib().or_mxfp4_dot(O.p(lin.data[r * cols // 2:], O._u8p), O.p(lin.exps[r * cols // 32:], O._u8p),
                                                  cols, O.p(q, O._i8p), O.p(s, O._f32p))
        tol = 1e-5
    else:
        want = x.astype(np.float64) @ oracle_dequant(lin).astype(np.float64).T
        # up to 8 tokens, and matrices under 4,096 rows: int8 hi/lo activations (about 15 bits);
        # 9..64 tokens of larger matrices (4104 x 768 here): the tensor-core GEMV's fp16 operands
        # (the weight and the activation each rounded to fp16, about 2^-12 of a product)
        tol = 1e-4 if ntok <= 8 or rows < 4096 else 1e-3
    scale = np.abs(want).max()
    assert np.abs(got - want).max() <= tol * scale + 1e-7, np.abs(got - want).max() / scale
    if ntok > 8 and fmt != A.HC_FMT_MXFP4 and rows >= 4096:
        # and no wait of the tensor-core GEMV ran out
        A.check(A.lib().hc_device_check(device.h))


def attention_ref(q, kc, vc, pos, window, sinks, scale):
    ntok, H, hd = q.shape
    KV = kc.shape[0]
    rep = H // KV
    out = np.zeros_like(q, dtype=np.float64)
    for t in range(ntok):
        P = pos + t
        lo = max(0, P - window + 1) if window else 0
        for h in range(H):
            k = kc[h // rep, lo:P + 1].astype(np.float64)
            v = vc[h // rep, lo:P + 1].astype(np.float64)
            s = k @ q[t, h].astype(np.float64) * scale
            m = s.max() if sinks is None else max(s.max(), sinks[h])
            e = np.exp(s - m)
            z = e.sum() + (0 if sinks is None else np.exp(sinks[h] - m))
            out[t, h] = (e / z) @ v
    return out


@pytest.mark.parametrize("H,KV,hd,window,sink", [(16, 8, 128, 0, False), (16, 4, 64, 0, False),
                                                   (64, 8, 64, 128, True), (64, 8, 64, 0, True), (8, 8, 128, 0, False)])
@pytest.mark.parametrize("ntok,pos", [(1, 0), (1, 300), (3, 1500), (5, 77)])
def test_attention(H, KV, hd, window, sink, ntok, pos):
    rng = np.random.default_rng(H * 7 + pos)
    cap = pos + ntok + 3
    q = rng.standard_normal((ntok, H, hd)).astype(np.float32)
    kc = rng.standard_normal((KV, cap, hd)).astype(np.float16)
    vc = rng.standard_normal((KV, cap, hd)).astype(np.float16)
    sinks = (rng.standard_normal(H) * 2).astype(np.float32) if sink else None
    scale = np.float32(synth.f16_values(synth.f16_bits(np.array([1 / np.sqrt(hd)], np.float32)))[0])
    tq, tk, tv = torch.from_numpy(q).cuda(), torch.from_numpy(kc.view(np.uint16).astype(np.int16)).cuda(), \
        torch.from_numpy(vc.view(np.uint16).astype(np.int16)).cuda()
    ts = torch.from_numpy(sinks).cuda() if sink else None
    to = torch.empty_like(tq)
    sc = np.array([scale], np.float32)
    A.check(A.lib().hc_attention_run(C.c_void_p(tq.data_ptr()), C.c_void_p(tk.data_ptr()), C.c_void_p(tv.data_ptr()),
                                     C.c_void_p(ts.data_ptr()) if sink else None, C.c_void_p(to.data_ptr()),
                                     ntok, H, KV, hd, pos, cap, window, sc.ctypes.data_as(C.POINTER(C.c_float)), None))
    got = to.cpu().numpy()
    want = attention_ref(q, kc, vc, pos, window, sinks, float(scale))
    assert np.abs(got - want).max() < 2e-5 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("ntok,pos,cap", [(1, 127, 128), (1, 300, 128), (1, 1000, 128), (3, 500, 130), (5, 77, 132)])
def test_attention_ring_window(ntok, pos, cap):
    # gpt-oss's sliding layers keep a ring of the window (gptoss StepInputs, build.go:291-326): the
    # key of position p at slot p mod cap; positions past the window have wrapped around
    H, KV, hd, window = 64, 8, 64, 128
    rng = np.random.default_rng(pos * 3 + ntok)
    q = rng.standard_normal((ntok, H, hd)).astype(np.float32)
    ring_k = rng.standard_normal((KV, cap, hd)).astype(np.float16)
    ring_v = rng.standard_normal((KV, cap, hd)).astype(np.float16)
    sinks = (rng.standard_normal(H) * 2).astype(np.float32)
    scale = np.float32(synth.f16_values(synth.f16_bits(np.array([1 / np.sqrt(hd)], np.float32)))[0])
    # the linear view the reference attends over: position p reads ring slot p mod cap
    P = pos + ntok
    lin_k = ring_k[:, np.arange(P) % cap]
    lin_v = ring_v[:, np.arange(P) % cap]
    tq = torch.from_numpy(q).cuda()
    tk = torch.from_numpy(ring_k.view(np.uint16).astype(np.int16)).cuda()
    tv = torch.from_numpy(ring_v.view(np.uint16).astype(np.int16)).cuda()
    ts = torch.from_numpy(sinks).cuda()
    to = torch.empty_like(tq)
    sc = np.array([scale], np.float32)
    A.check(A.lib().hc_attention_run(C.c_void_p(tq.data_ptr()), C.c_void_p(tk.data_ptr()), C.c_void_p(tv.data_ptr()),
                                     C.c_void_p(ts.data_ptr()), C.c_void_p(to.data_ptr()), ntok, H, KV, hd, pos, cap,
                                     window, sc.ctypes.data_as(C.POINTER(C.c_float)), None))
    want = attention_ref(q, lin_k, lin_v, pos, window, sinks, float(scale))
    got = to.cpu().numpy()
    assert np.abs(got - want).max() < 2e-5 * max(1.0, np.abs(want).max())


def test_attention_ring_too_small_is_an_error():
    # a ring of exactly the window cannot hold a 3-token step's own rows
    z = torch.zeros(1 << 16, device="cuda")
    p = C.c_void_p(z.data_ptr())
    sc = np.array([0.125], np.float32)
    with pytest.raises(hb.HcError, match="ring"):
        A.check(A.lib().hc_attention_run(p, p, p, None, p, 3, 8, 8, 64, 500, 128, 128,
                                         sc.ctypes.data_as(C.POINTER(C.c_float)), None))


def test_argmax_first_of_equal():
    v = np.full((3, 151936), -5.0, np.float32)
    v[0, [7, 99, 151935]] = 3.0       # a tie: the first wins
    v[1, 151935] = 1.0
    v[2, :] = -0.0
    v[2, 10] = 0.0                    # +0 and -0 are equal: index 0 wins
    h = torch.from_numpy(synth.f16_bits(v).astype(np.int16)).cuda()
    out = torch.empty(3, dtype=torch.int32, device="cuda")
    A.check(A.lib().hc_argmax_run(C.c_void_p(h.data_ptr()), 3, 151936, C.c_void_p(out.data_ptr()), None))
    assert out.cpu().tolist() == [7, 151935, 0]


def test_route_matches_oracle():
    rng = np.random.default_rng(9)
    rows, n, k = 33, 32, 4
    logits = rng.standard_normal((rows, n)).astype(np.float32)
    logits[0, [3, 9, 20, 21]] = 4.0  # ties
    tl = torch.from_numpy(logits).cuda()
    ti = torch.empty((rows, k), dtype=torch.int32, device="cuda")
    tw = torch.empty((rows, k), dtype=torch.float32, device="cuda")
    A.check(A.lib().hc_route_run(C.c_void_p(tl.data_ptr()), rows, n, k, C.c_void_p(ti.data_ptr()), C.c_void_p(tw.data_ptr()), None))
    gi, gw = ti.cpu().numpy(), tw.cpu().numpy()
    for r in range(rows):
        idx, w = np.zeros(k, np.int32), np.zeros(k, np.float32)
        lr = np.ascontiguousarray(logits[r])
        O.lib().or_route(O.p(lr, O._f32p), n, k, 1, O.p(idx, O._i32p), O.p(w, O._f32p))
        assert gi[r].tolist() == idx.tolist()
        assert np.allclose(gw[r], w, rtol=1e-6, atol=0)
