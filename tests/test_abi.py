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
    src = open(os.path.join(ROOT, "include", "hwnpu_cuda.h")).read()
    return sorted(set(re.findall(r"HC_API\s+[\w\s\*]*?\b(hc_\w+)\s*\(", src)))


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


def test_descriptor_layout_matches_header():
    # the C struct sizes the Go/purego side would mirror
    assert C.sizeof(A.LinearDesc) == 56
    assert C.sizeof(A.SessionOpts) == 24
    assert C.sizeof(A.Stats) == 48
    assert A.ModelDesc.head.offset % 8 == 0
