"""hc_attention_run_static (the attention entry point that allocates nothing) against
hc_attention_run, through the C ABI, on two calls in a row with different shapes. The file sorts
last so that it also runs after every other test has used the device."""
import ctypes as C

import numpy as np
import pytest

from hwnpu_b200 import _abi as A
from hwnpu_b200 import synth

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

# the attention tests' tolerance (tests/test_gpu_kernels.py): relative to the largest output
TOL = 2e-5


def _case(rng, ntok, H, KV, hd, pos, window, sink):
    cap = pos + ntok + 3
    q = rng.standard_normal((ntok, H, hd)).astype(np.float32)
    kc = rng.standard_normal((KV, cap, hd)).astype(np.float16)
    vc = rng.standard_normal((KV, cap, hd)).astype(np.float16)
    sinks = (rng.standard_normal(H) * 2).astype(np.float32) if sink else None
    scale = np.array(synth.f16_values(synth.f16_bits(np.array([1 / np.sqrt(hd)], np.float32))), np.float32)
    dev = dict(q=torch.from_numpy(q).cuda(),
               k=torch.from_numpy(kc.view(np.uint16).astype(np.int16)).cuda(),
               v=torch.from_numpy(vc.view(np.uint16).astype(np.int16)).cuda(),
               s=torch.from_numpy(sinks).cuda() if sink else None)
    return dict(dev=dev, ntok=ntok, H=H, KV=KV, hd=hd, pos=pos, cap=cap, window=window, scale=scale)


def _run(fn, c, out):
    d = c["dev"]
    A.check(fn(C.c_void_p(d["q"].data_ptr()), C.c_void_p(d["k"].data_ptr()), C.c_void_p(d["v"].data_ptr()),
               C.c_void_p(d["s"].data_ptr()) if d["s"] is not None else None, C.c_void_p(out.data_ptr()),
               c["ntok"], c["H"], c["KV"], c["hd"], c["pos"], c["cap"], c["window"],
               c["scale"].ctypes.data_as(C.POINTER(C.c_float)), None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_static_matches_allocating_entry_twice():
    # Both entry points run the same kernels with the same splits, so their outputs agree bit for
    # bit. The large gpt-oss-like case (about 1.3 MB of partials) runs first and leaves stale
    # partials in every part of the scratch the small C2 case (about 130 KB) then reads; the large
    # case runs again after it. Equality on every call shows that nothing in the scratch needs to
    # start at zero.
    rng = np.random.default_rng(2024)
    big = _case(rng, 5, 64, 8, 64, 300, 128, True)     # gpt-oss-like: sinks, sliding window
    small = _case(rng, 1, 16, 8, 128, 1100, 0, False)  # the C2 decode shape
    for c in (big, small, big):
        ref = _run(A.lib().hc_attention_run, c, torch.empty_like(c["dev"]["q"]))
        got = _run(A.lib().hc_attention_run_static, c, torch.empty_like(c["dev"]["q"]))
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert np.abs(got - ref).max() <= TOL * max(1.0, np.abs(ref).max())


def test_static_rejects_oversized_scratch():
    c = _case(np.random.default_rng(1), 1, 8, 8, 64, 0, 0, False)
    d = c["dev"]
    dummy = C.c_void_p(d["q"].data_ptr())
    sc = c["scale"].ctypes.data_as(C.POINTER(C.c_float))
    # 64 tokens x 64 heads x head_dim 128: 33.5 MB of partials alone
    err = A.lib().hc_attention_run_static(dummy, dummy, dummy, None, dummy, 64, 64, 8, 128, 0, 64, 0, sc, None)
    assert err, "a call beyond the static scratch must fail"
    msg = C.cast(err, C.c_char_p).value.decode()
    A.lib().hc_free_error(err)
    assert "static limit" in msg
