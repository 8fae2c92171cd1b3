"""Host-side mirror of the reference interfaces this engine plugs into.

- Provider / Device / Buffer: backend.Provider, backend.Device, backend.Buffer
  (internal/backend/backend.go:13-67) over hc_device_* / hc_buf_*.
- Session: chat.session + chat.tokenSession (internal/chat/session.go:9-32) over hc_session_*,
  one sequence slot per Session view (Seq) or many (step_batch, the ragged batch).

Every method calls the C ABI; errors come back as HcError, as the Go side's error values.
"""

import ctypes as C

import numpy as np

from . import _abi as A
from .synth import f16_values


class Provider:
    """backend.Provider for CUDA devices (backends.go:14-19 registers one per backend)."""

    name = "cuda"

    def enumerate(self):
        n = C.c_uint32()
        A.check(A.lib().hc_device_count(C.byref(n)))
        return list(range(n.value))

    def open(self, index=0):
        return Device(index)


class Device:
    def __init__(self, index=0):
        h = C.c_void_p()
        A.check(A.lib().hc_device_open(index, C.byref(h)))
        self.h = h

    def info(self, key):
        need = C.c_size_t()
        A.check(A.lib().hc_device_info(self.h, key, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        A.check(A.lib().hc_device_info(self.h, key, buf, need.value, C.byref(need)))
        return buf.value.decode()

    def alloc_buffer(self, size, kind=A.HC_BUF_DEVICE):
        return Buffer(self, size, kind)

    def load_model(self, model):
        return LoadedModel(self, model)

    def close(self):
        if self.h:
            A.lib().hc_device_free(self.h)
            self.h = None


class Buffer:
    """backend.Buffer: Bytes (a host view), SyncToDevice, SyncFromDevice, Close."""

    def __init__(self, dev, size, kind):
        h = C.c_void_p()
        A.check(A.lib().hc_buf_alloc(dev.h, size, kind, C.byref(h)))
        self.h, self.size = h, size
        p = C.c_void_p()
        A.check(A.lib().hc_buf_map(h, C.byref(p)))
        self._view = np.ctypeslib.as_array((C.c_uint8 * size).from_address(p.value)) if size else np.zeros(0, np.uint8)

    def bytes(self):
        return self._view

    def address(self):
        return A.lib().hc_buf_address(self.h)

    def sync_to_device(self, off=0, n=None):
        A.check(A.lib().hc_buf_sync(self.h, A.HC_SYNC_TO_DEVICE, off, self.size - off if n is None else n))

    def sync_from_device(self, off=0, n=None):
        A.check(A.lib().hc_buf_sync(self.h, A.HC_SYNC_FROM_DEVICE, off, self.size - off if n is None else n))

    def close(self):
        if self.h:
            A.lib().hc_buf_free(self.h)
            self.h = None


class LoadedModel:
    def __init__(self, dev, model):
        self.dev, self.model = dev, model
        h = C.c_void_p()
        A.check(A.lib().hc_model_load(dev.h, C.byref(model.desc()), C.byref(h)))
        self.h = h

    @property
    def weight_bytes(self):
        return A.lib().hc_model_weight_bytes(self.h)

    def session(self, max_context, max_seqs=1, max_step=8, kv_format=A.HC_KV_F16, page_size=16, graphs=True):
        flags = 0 if graphs else A.HC_SESSION_NO_GRAPH
        return Session(self, max_context, max_seqs, max_step, kv_format, page_size, flags)

    def close(self):
        if self.h:
            A.lib().hc_model_free(self.h)
            self.h = None


def _i32(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def _u16(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint16))


class Session:
    """decode.Session / chat.tokenSession over a device-resident KV cache of max_seqs slots."""

    def __init__(self, lm, max_context, max_seqs, max_step, kv_format, page_size, flags):
        self.lm = lm
        self.vocab = lm.model.cfg.vocab
        o = A.SessionOpts(max_context, max_seqs, max_step, kv_format, page_size, flags)
        h = C.c_void_p()
        A.check(A.lib().hc_session_new(lm.h, C.byref(o), C.byref(h)))
        self.h, self.max_context, self.max_seqs, self.max_step = h, max_context, max_seqs, max_step

    # -- tokenSession ----------------------------------------------------------------------
    def step_batch(self, seqs, token_lists, all_rows=False, want_logits=True, timeout_ms=0):
        """hc_step over several sequences: returns (logits fp16 bits [rows][vocab] or None,
        argmax [rows]). rows: each sequence's last token, or every token with all_rows."""
        seqs = np.asarray(seqs, np.int32)
        counts = np.asarray([len(t) for t in token_lists], np.int32)
        toks = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int32) for t in token_lists]))
        rows = int(counts.sum()) if all_rows else len(seqs)
        logits = np.empty((rows, self.vocab), np.uint16) if want_logits else None
        am = np.empty(rows, np.int32)
        state = C.c_int32()
        A.check(A.lib().hc_step(self.h, _i32(seqs), _i32(counts), _i32(toks), len(seqs),
                                A.HC_STEP_ALL_ROWS if all_rows else 0,
                                _u16(logits) if logits is not None else None, _i32(am), timeout_ms,
                                C.byref(state)))
        if state.value == A.HC_STATE_TIMEOUT:
            raise TimeoutError("hc_step timed out")
        return logits, am

    def step_tokens(self, toks, seq=0, all_rows=False):
        """tokenSession.StepTokens: the logits (float32) after the last token (every token with
        all_rows), from the fp16 the step writes."""
        logits, _ = self.step_batch([seq], [toks], all_rows=all_rows)
        return f16_values(logits) if all_rows else f16_values(logits[0])

    def greedy(self, toks, seq=0):
        """StepTokens that keeps only the greedy choice after the last token."""
        _, am = self.step_batch([seq], [toks], want_logits=False)
        return int(am[0])

    def speculate_tokens(self, toks, seq=0, want_logits=False):
        """tokenSession.SpeculateTokens with greedy acceptance (chat/engine.go:1044-1058), on the
        device: returns (kept, next token, logits of the last kept row or None)."""
        toks = np.ascontiguousarray(toks, np.int32)
        kept, nxt, state = C.c_int32(), C.c_int32(), C.c_int32()
        logits = np.empty(self.vocab, np.uint16) if want_logits else None
        A.check(A.lib().hc_speculate(self.h, seq, _i32(toks), len(toks), C.byref(kept), C.byref(nxt),
                                     _u16(logits) if logits is not None else None, 0, C.byref(state)))
        return kept.value, nxt.value, (f16_values(logits) if logits is not None else None)

    def generate(self, first, n, seq=0, timeout_ms=0):
        """Greedy generation of n tokens on the device from `first` (hc_generate)."""
        out = np.empty(n, np.int32)
        state = C.c_int32()
        A.check(A.lib().hc_generate(self.h, seq, int(first), n, _i32(out), timeout_ms, C.byref(state)))
        if state.value == A.HC_STATE_TIMEOUT:
            raise TimeoutError("hc_generate timed out")
        return out

    def stream(self):
        """The session's cudaStream_t as an integer handle."""
        p = C.c_void_p()
        A.check(A.lib().hc_session_stream(self.h, C.byref(p)))
        return p.value or 0

    # -- session ---------------------------------------------------------------------------
    def pos(self, seq=0):
        p = C.c_int32()
        A.check(A.lib().hc_seq_pos(self.h, seq, C.byref(p)))
        return p.value

    def reset(self, seq=0):
        A.check(A.lib().hc_seq_reset(self.h, seq))

    def truncate(self, length, seq=0):
        A.check(A.lib().hc_seq_truncate(self.h, seq, length))

    def export_rows(self, start, n, seq=0):
        need = C.c_uint64()
        A.check(A.lib().hc_seq_export_rows(self.h, seq, start, n, None, 0, C.byref(need)))
        out = np.empty(need.value, np.uint8)
        A.check(A.lib().hc_seq_export_rows(self.h, seq, start, n, out.ctypes.data_as(C.c_void_p), out.nbytes, C.byref(need)))
        return out

    def import_rows(self, start, n, rows, seq=0):
        rows = np.ascontiguousarray(rows, np.uint8)
        A.check(A.lib().hc_seq_import_rows(self.h, seq, start, n, rows.ctypes.data_as(C.c_void_p), rows.nbytes))

    def stats(self):
        s = A.Stats()
        A.check(A.lib().hc_stats_get(self.h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in A.Stats._fields_}

    def close(self):
        if self.h:
            A.lib().hc_session_free(self.h)
            self.h = None
