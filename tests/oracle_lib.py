"""ctypes binding of oracle/liboracle.so, the CPU restatement of the reference path.

Test infrastructure: only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use it.
"""

import ctypes as C
import os

import numpy as np

from hwnpu_b200 import _abi as A

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PATH = os.path.join(ROOT, "oracle", "liboracle.so")
_o = None

_f32p, _u8p, _u16p, _i32p, _i8p = (C.POINTER(C.c_float), C.POINTER(C.c_uint8), C.POINTER(C.c_uint16),
                                   C.POINTER(C.c_int32), C.POINTER(C.c_int8))
SIG = {
    "or_f16_bits": (C.c_uint16, [C.c_float]),
    "or_f16_value": (C.c_float, [C.c_uint16]),
    "or_exp": (C.c_float, [C.c_float]),
    "or_synth_uniform": (None, [C.c_char_p, _f32p, C.c_uint64]),
    "or_synth_normal": (None, [C.c_uint64, C.c_char_p, _f32p, _f32p, C.c_uint64]),
    "or_synth_tokens": (None, [C.c_uint64, C.c_int32, _i32p, C.c_uint64]),
    "or_f32_to_f16_n": (None, [_f32p, _u16p, C.c_uint64]),
    "or_quantize_linear": (None, [_f32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int32, C.c_int32, _u8p, _u16p]),
    "or_dequant_linear": (None, [_u8p, _u16p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int32, _f32p]),
    "or_dequant_int4_asym": (None, [_u8p, _u16p, _u16p, C.c_uint32, C.c_uint32, _f32p]),
    "or_quantize_int4_asym": (None, [_f32p, C.c_uint32, C.c_uint32, _u8p, _u16p, _u16p]),
    "or_mxfp4_nearest": (C.c_uint8, [C.c_double]),
    "or_mxfp4_encode": (None, [_f32p, C.c_uint32, _u8p, _u8p]),
    "or_mxfp4_dequant": (None, [_u8p, _u8p, C.c_uint32, _f32p]),
    "or_mxfp4_quantize": (None, [_f32p, C.c_uint32, _i8p, _f32p]),
    "or_mxfp4_dot": (C.c_float, [_u8p, _u8p, C.c_uint32, _i8p, _f32p]),
    "or_route": (None, [_f32p, C.c_int32, C.c_int32, C.c_int32, _i32p, _f32p]),
    "or_merge_new": (C.c_void_p, [C.c_int32, C.c_int32]),
    "or_merge_free": (None, [C.c_void_p]),
    "or_merge_add": (None, [C.c_void_p, _f32p, _f32p, _f32p]),
    "or_merge_add_sink": (None, [C.c_void_p, _f32p, C.c_int32]),
    "or_merge_result": (None, [C.c_void_p, _f32p]),
    "or_gemm_nt": (None, [C.c_int32, C.c_int32, C.c_int32, _f32p, _f32p, _f32p, C.c_int32]),
    "or_argmax": (C.c_int32, [_f32p, C.c_int32]),
    "or_argmax_f16": (C.c_int32, [_u16p, C.c_int32]),
    "or_model_new": (C.c_void_p, [C.POINTER(A.ModelDesc), C.c_int32]),
    "or_model_free": (None, [C.c_void_p]),
    "or_session_new": (C.c_void_p, [C.c_void_p, C.c_int32]),
    "or_session_new_kv": (C.c_void_p, [C.c_void_p, C.c_int32, C.c_int32]),
    "or_session_free": (None, [C.c_void_p]),
    "or_session_pos": (C.c_int32, [C.c_void_p]),
    "or_step": (C.c_int32, [C.c_void_p, _i32p, C.c_int32, C.c_int32, _u16p]),
    "or_speculate": (C.c_int32, [C.c_void_p, _i32p, C.c_int32, _i32p, _u16p]),
    "or_truncate": (None, [C.c_void_p, C.c_int32]),
    "or_page_write": (None, [_i8p, _u16p, C.c_int32, _f32p, C.c_int32]),
}


def lib():
    global _o
    if _o is None:
        L = C.CDLL(PATH)
        for k, (r, a) in SIG.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        _o = L
    return _o


def p(a, t):
    return a.ctypes.data_as(t)


def _row_blocks(rows, fn, block=256):
    """Runs fn(r0, r1) over row blocks on the host's threads (ctypes releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    spans = [(r, min(rows, r + block)) for r in range(0, rows, block)]
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        list(ex.map(lambda s: fn(*s), spans))


class OracleGen:
    """synth.Model's generator on the oracle's side (or_synth_*, or_quantize_*, or_mxfp4_encode):
    the same values and bytes as the product library's, with no call into libhwnpu_cuda.so."""

    @staticmethod
    def normal(seed, name, n, std):
        out = np.empty(n, np.float32)
        sd = np.array([std], np.float32)
        lib().or_synth_normal(seed, name.encode(), p(sd, _f32p), p(out, _f32p), n)
        return out

    @staticmethod
    def tokens(seed, vocab, n):
        out = np.empty(n, np.int32)
        lib().or_synth_tokens(seed, vocab, p(out, _i32p), n)
        return out

    @staticmethod
    def f16_bits(x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.shape, np.uint16)
        lib().or_f32_to_f16_n(p(x, _f32p), p(out, _u16p), x.size)
        return out

    @staticmethod
    def quantize(w, fmt, search=False):
        from hwnpu_b200.synth import Linear

        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        L = lib()
        if fmt in (A.HC_FMT_INT8_ROW, A.HC_FMT_INT4_SYM_G32):
            bits, blk = (8, cols) if fmt == A.HC_FMT_INT8_ROW else (4, 32)
            per = cols // blk
            data = np.empty(rows * cols * bits // 8, np.uint8)
            sc = np.empty(rows * per, np.uint16)
            rb = cols * bits // 8

            def run(r0, r1):
                L.or_quantize_linear(p(w[r0:r1], _f32p), r1 - r0, cols, 0 if bits == 8 else 32, bits, int(search),
                                     p(data[r0 * rb:], _u8p), p(sc[r0 * per:], _u16p))
            _row_blocks(rows, run)
            return Linear(fmt, rows, cols, data, scales=sc)
        if fmt == A.HC_FMT_INT4_ASYM_G32:
            data = np.empty(rows * cols // 2, np.uint8)
            sc = np.empty(rows * cols // 32, np.uint16)
            z = np.empty(rows * cols // 32, np.uint16)

            def run(r0, r1):
                L.or_quantize_int4_asym(p(w[r0:r1], _f32p), r1 - r0, cols, p(data[r0 * cols // 2:], _u8p),
                                        p(sc[r0 * cols // 32:], _u16p), p(z[r0 * cols // 32:], _u16p))
            _row_blocks(rows, run)
            return Linear(fmt, rows, cols, data, scales=sc, zeros=z)
        if fmt == A.HC_FMT_MXFP4:
            data = np.empty(rows * cols // 2, np.uint8)
            e = np.empty(rows * cols // 32, np.uint8)

            def run(r0, r1):
                for r in range(r0, r1):
                    L.or_mxfp4_encode(p(w[r], _f32p), cols, p(data[r * cols // 2:], _u8p), p(e[r * cols // 32:], _u8p))
            _row_blocks(rows, run, block=64)
            return Linear(fmt, rows, cols, data, exps=e)
        raise ValueError(f"format {fmt}")


class OracleSession:
    """decode.Session on the CPU interpreter for a synth.Model."""

    def __init__(self, model, max_context, threads=0, kv_format=A.HC_KV_F16, share=None):
        """share: another OracleSession of the same model whose (large) float32 weights this one
        uses instead of its own copy."""
        self.model = model
        self.vocab = model.cfg.vocab
        self.owner = share is None
        self.m = lib().or_model_new(C.byref(model.desc()), threads or os.cpu_count()) if share is None else share.m
        assert self.m, "oracle: model not supported"
        self.s = lib().or_session_new_kv(self.m, max_context, kv_format)
        assert self.s, "oracle: kv format not supported"

    def step(self, toks, all_rows=False):
        toks = np.ascontiguousarray(toks, np.int32)
        rows = len(toks) if all_rows else 1
        out = np.empty((rows, self.vocab), np.uint16)
        rc = lib().or_step(self.s, p(toks, _i32p), len(toks), int(all_rows), p(out, _u16p))
        assert rc == 0, "oracle step failed"
        return out

    def speculate(self, toks):
        toks = np.ascontiguousarray(toks, np.int32)
        nxt = np.zeros(1, np.int32)
        out = np.empty(self.vocab, np.uint16)
        kept = lib().or_speculate(self.s, p(toks, _i32p), len(toks), p(nxt, _i32p), p(out, _u16p))
        return kept, int(nxt[0]), out

    def pos(self):
        return lib().or_session_pos(self.s)

    def truncate(self, n):
        lib().or_truncate(self.s, n)

    def close(self):
        if self.s:
            lib().or_session_free(self.s)
            if self.owner:
                lib().or_model_free(self.m)
            self.s = self.m = None
