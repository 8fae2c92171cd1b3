"""The C ABI without a GPU: the library loads, exports what include/hwnpu_cuda.h declares, and
its host-side logic (errors, fault specs, device enumeration) behaves."""

import ctypes as C
import os
import re

import numpy as np
import pytest

import hwnpu_b200 as hb
from hwnpu_b200 import _abi as A

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    """Every hc_* entry point the headers under include/ declare (the product ABI, hwnpu_cuda.h,
    and the test and benchmark helpers of hwnpu_cuda_synth.h)."""
    names = set()
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            names |= set(re.findall(r"HC_API\s+[\w\s\*]*?\b(hc_\w+)\s*\(", src))
    return sorted(names)


def test_synth_helpers_are_outside_the_product_header():
    src = open(os.path.join(ROOT, "include", "hwnpu_cuda.h")).read()
    assert "hc_synth_" not in re.sub(r"/\*.*?\*/", "", src, flags=re.S)


def test_every_declared_symbol_is_exported_and_bound():
    names = declared()
    assert len(names) >= 39
    lib = C.CDLL(A.lib_path())
    for n in names:
        assert hasattr(lib, n), f"{n} not exported"
    assert set(names) == set(A.SIGNATURES), set(names) ^ set(A.SIGNATURES)


def test_abi_version():
    assert A.lib().hc_abi() == A.HC_ABI


def test_device_count_without_gpu_is_clean():
    n = C.c_uint32(99)
    err = A.lib().hc_device_count(C.byref(n))
    if err:  # no driver: an error string, freed
        msg = C.cast(err, C.c_char_p).value.decode()
        A.lib().hc_free_error(err)
        assert "cuda" in msg
    else:
        assert n.value >= 0


def test_error_protocol_and_fault_specs():
    with pytest.raises(hb.HcError, match="unknown point"):
        A.check(A.lib().hc_set_fault(b"disk:1"))
    with pytest.raises(hb.HcError, match="at least 1"):
        A.check(A.lib().hc_set_fault(b"step:0"))
    A.check(A.lib().hc_set_fault(b"step:2"))
    A.check(A.lib().hc_set_fault(b""))


def test_null_arguments_are_errors_not_crashes():
    with pytest.raises(hb.HcError):
        A.check(A.lib().hc_model_load(None, None, None))
    with pytest.raises(hb.HcError):
        A.check(A.lib().hc_step(None, None, None, None, 0, 0, None, None, 0, None))
    with pytest.raises(hb.HcError):
        A.check(A.lib().hc_quantize_linear(None, 1, 6, 0, 5, 0, None, None))


def test_synth_is_seeded_and_thread_count_free():
    a = hb.synth.normal(0, "model.layers.0.self_attn.q_proj.weight", 3 << 20, 0.02)
    b = hb.synth.normal(0, "model.layers.0.self_attn.q_proj.weight", 3 << 20, 0.02)
    c = hb.synth.normal(1, "model.layers.0.self_attn.q_proj.weight", 1000, 0.02)
    assert np.array_equal(a, b) and not np.array_equal(a[:1000], c)
    assert abs(a.std() - 0.02) < 1e-4 and abs(a.mean()) < 1e-4
    t = hb.synth.tokens(1, 151936, 10000)
    assert t.min() >= 0 and t.max() < 151936


def test_oracle_generator_equals_the_library_generator():
    # the CPU arm of the benchmark builds its weights with the oracle's generator and quantisers
    # (no call into libhwnpu_cuda.so); they must be the GPU arm's bytes exactly
    import oracle_lib as O

    for n in (7, 1 << 20, (3 << 20) + 5):
        a = hb.synth.normal(3, "model.layers.1.mlp.up_proj.weight", n, 0.02)
        b = O.OracleGen.normal(3, "model.layers.1.mlp.up_proj.weight", n, 0.02)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), n
    assert np.array_equal(hb.synth.tokens(9, 32000, 4097), O.OracleGen.tokens(9, 32000, 4097))
    x = hb.synth.normal(4, "x", 5000, 3.0)
    assert np.array_equal(hb.synth.f16_bits(x), O.OracleGen.f16_bits(x))
    w = hb.synth.normal(5, "w", 300 * 512, 0.02).reshape(300, 512)
    for fmt in (A.HC_FMT_INT8_ROW, A.HC_FMT_INT4_SYM_G32, A.HC_FMT_INT4_ASYM_G32, A.HC_FMT_MXFP4):
        lp, op = hb.synth.Linear.quantize(w, fmt), O.OracleGen.quantize(w, fmt)
        for k in ("data", "scales", "zeros", "exps"):
            u, v = getattr(lp, k), getattr(op, k)
            assert (u is None) == (v is None), (fmt, k)
            if u is not None:
                assert np.array_equal(u, v), (fmt, k)
    cfg = hb.synth.Config("gen-check", 1, 256, 512, 4, 2, 64, 300, A.HC_FMT_INT4_ASYM_G32, tied=True, qk_norm=True)
    m1 = hb.synth.Model(cfg, seed=2, norm_std=0.1)
    m2 = hb.synth.Model(cfg, seed=2, norm_std=0.1, gen=O.OracleGen)
    assert np.array_equal(m1.head.data, m2.head.data) and np.array_equal(m1.head.zeros, m2.head.zeros)
    assert np.array_equal(m1.layers[0]["q_norm"], m2.layers[0]["q_norm"])


def test_descriptor_layout_matches_header():
    # the C struct sizes the Go/purego side would mirror
    assert C.sizeof(A.LinearDesc) == 56
    assert C.sizeof(A.SessionOpts) == 24
    assert C.sizeof(A.Stats) == 48
    assert A.ModelDesc.head.offset % 8 == 0
