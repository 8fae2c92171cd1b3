#!/usr/bin/env python
"""Decode benchmark of the B200 engine on BASELINE.json's headline metric: decode tokens/s of the
64-sequence ragged batch (configs[4], C5) at 1/2/4/8 GPUs, with the batch-1 figures of the 1.7B
model (configs[1], C2) nested under "bs1"; % of the HBM roofline for both.

Default line (no --workload): C5 continuous-batched ragged decode of the C2 model over the paged
int8 KV cache. 64 sequences with contexts drawn uniform on 128..8192 (seed 2) are sharded round
robin over the ranks (weights replicated, no collective on the path); a step is one hc_step call
over every slot of the rank (each slot's next token, or the 512-id prompt of a new sequence that
took a finished one's slot). W untimed steps, then exactly K timed steps. value: the decoded tokens
of all ranks / the slowest rank's device time (the sum of the call's chunk graphs, CUDA events);
"scaling": "strong" (the 64 sequences are the job whatever N). e2e: the same tokens over CUDA
events around the whole host loop (token lists in from host memory, greedy choices out).
bs1: C2 greedy decode after a 1024-id prompt on every rank (its own sequence), K tokens of the
device-resident loop (hc_generate) and of the per-token public call (hc_step) in passes of 256
from the prompt (context 1024-1280).

--impl reference times the reference path's CPU restatement (oracle/: the Go path cannot run
here) on the host's cores for the same metric: weights built by the oracle's own generator (no
call into libhwnpu_cuda.so), per-token decode costs sampled at two contexts and the prefill rate,
extrapolated to the same C5 schedule; rank 0 only.

Workloads c2 / c1 (bs1 lines), c3 (the MoE model at batch 1 and 16), c4 (speculative), linear
(one GEMV) remain as --workload.
"""

import argparse
import dataclasses
import hashlib
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (bs1, 64 ragged) at 1/2/4/8 B200; % HBM roofline"
PROMPT = 1024
PASS = 256
C5_SEQS, C5_OWED, C5_NEW_PROMPT = 64, 128, 512
# C2's paged int8 KV: int8 K and V rows + fp16 page scales, per position and layer, all layers
C5_KV_POS = 28 * (8 * 128 * 2 + 2 * 8 * 2 / 16)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_info():
    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return os.cpu_count() or 1, model


class Clocks:
    """SM clock and clock-event (throttle) reasons sampled through NVML every 10 ms while running."""

    def __init__(self, gpu):
        self.gpu, self.samples, self.run, self.th = gpu, [], False, None
        self.mx = None

    def start(self):
        try:
            import pynvml as N

            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByIndex(self.gpu)
            self.mx = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            names = {N.nvmlClocksThrottleReasonHwSlowdown: "hw_slowdown",
                     N.nvmlClocksThrottleReasonHwThermalSlowdown: "hw_thermal_slowdown",
                     N.nvmlClocksThrottleReasonSwThermalSlowdown: "sw_thermal_slowdown",
                     N.nvmlClocksThrottleReasonSwPowerCap: "sw_power_cap"}

            def loop():
                while self.run:
                    try:
                        sm = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
                        r = N.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                        self.samples.append((sm, [v for k, v in names.items() if r & k]))
                    except Exception:
                        pass
                    time.sleep(0.01)

            self.run = True
            self.th = threading.Thread(target=loop, daemon=True)
            self.th.start()
        except Exception:
            self.run = False

    def stop(self):
        if not self.run:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        self.run = False
        self.th.join()
        sm = sorted(s for s, _ in self.samples)
        reasons = sorted({r for _, rs in self.samples for r in rs})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": self.mx, "reasons": reasons,
                "samples": len(sm), "source": "NVML every 10 ms during the timed region"}


def c5_contexts():
    import numpy as np

    return np.random.default_rng(2).integers(128, 8192, size=C5_SEQS, endpoint=True)


class C5Schedule:
    """The C5 batch of one rank: each slot's owed decode steps (sequence i starts with 128 - 2 i,
    so they finish at different steps) and, once done, a new sequence with a 512-id prompt in its
    slot. Both arms walk the same schedule."""

    def __init__(self, mine):
        self.mine = list(mine)
        self.owed = [C5_OWED - 2 * g for g in self.mine]
        self.seed = [1000 + g * 64 for g in self.mine]
        ctx = c5_contexts()
        self.ctx = [int(ctx[g]) for g in self.mine]  # positions each slot holds

    def step(self):
        """Advances one step: returns per slot ("decode", None) or ("prompt", seed of the new ids)."""
        out = []
        for i in range(len(self.mine)):
            if self.owed[i] <= 0:
                self.seed[i] += 1
                self.owed[i] = C5_OWED
                self.ctx[i] = 0
                out.append(("prompt", self.seed[i]))
                self.ctx[i] += C5_NEW_PROMPT
            else:
                out.append(("decode", None))
                self.ctx[i] += 1
            self.owed[i] -= 1
        return out


# ---- the CPU side: the oracle (the reference path restated) on the host's cores ----------------
class CpuSample:
    """The oracle's C2 costs on this host, a bounded sample: the weights built by the oracle's own
    generator (the GPU arm's bytes, tests/test_abi.py checks it; libhwnpu_cuda.so is never
    mapped), a prefill of a 1024-id prompt timed (tokens/s of prompt reading), and greedy decode
    steps timed at two contexts (after a 64-id prompt and after the 1024-id one), so that a decode
    token's cost is modelled as t0 + t1 * context for the paged int8 cache (C5) or the fp16 cache
    (bs1)."""

    def __init__(self, threads, kv_format, decode_steps=3):
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import numpy as np

        import oracle_lib as O
        from hwnpu_b200 import _abi as A
        from hwnpu_b200 import synth

        self.threads = threads
        t0 = time.perf_counter()
        model = synth.Model(synth.C2, seed=0, gen=O.OracleGen)
        self.build_s = time.perf_counter() - t0
        ctx_cap = PROMPT + decode_steps + 8
        short = O.OracleSession(model, 64 + decode_steps + 8, threads=threads, kv_format=kv_format)
        long_ = O.OracleSession(model, ctx_cap, threads=threads, kv_format=kv_format, share=short)

        def decode(sess, prompt_len, seed):
            toks = O.OracleGen.tokens(seed, synth.C2.vocab, prompt_len)
            a = time.perf_counter()
            logits = sess.step(toks)[0]
            pre = time.perf_counter() - a
            a = time.perf_counter()
            for _ in range(decode_steps):
                t = O.lib().or_argmax_f16(O.p(logits, O._u16p), synth.C2.vocab)
                logits = sess.step([t])[0]
            return pre, (time.perf_counter() - a) / decode_steps

        _, d_short = decode(short, 64, 1)
        pre, d_long = decode(long_, PROMPT, 1)
        long_.close()
        short.close()
        self.prefill_tok_s = PROMPT / pre
        self.c_short, self.c_long = 64 + decode_steps / 2.0, PROMPT + decode_steps / 2.0
        self.t1 = max(0.0, (d_long - d_short) / (self.c_long - self.c_short))
        self.t0 = d_short - self.t1 * self.c_short
        self.d_short, self.d_long = d_short, d_long
        self.wall_s = time.perf_counter() - t0
        self.kv = "paged int8" if kv_format == A.HC_KV_INT8_PAGED else "fp16"

    def token_s(self, ctx):
        return self.t0 + self.t1 * ctx

    def describe(self):
        return (f"oracle C2 ({self.kv} KV) on {self.threads} threads: prefill of a {PROMPT}-id prompt "
                f"{self.prefill_tok_s:.1f} tok/s; greedy decode {1e3 * self.d_short:.0f} ms/token at context "
                f"{self.c_short:.0f} and {1e3 * self.d_long:.0f} ms/token at {self.c_long:.0f} "
                f"(cost modelled as linear in the context); {self.wall_s:.0f} s of CPU work")


def cpu_c5(sample, world, steps):
    """tokens/s of the C5 schedule on the CPU (every rank's slots one after another on one host):
    each decoded token at its context by the linear model, each new sequence's prompt at the
    prefill rate; extrapolated from the sample."""
    from hwnpu_b200 import replicas

    total_s, dec = 0.0, 0
    for r in range(world):
        sch = C5Schedule(replicas.shard(C5_SEQS, r, world))
        for _ in range(steps):
            for i, (kind, _) in enumerate(sch.step()):
                if kind == "prompt":
                    total_s += C5_NEW_PROMPT / sample.prefill_tok_s
                else:
                    total_s += sample.token_s(sch.ctx[i])
                dec += 1
    return dec / total_s


def cpu_c3(threads):
    """The oracle's C3 decode rate on this host, a bounded sample: the model's layer shapes on 2 of
    its 24 layers (vocabulary 201088, weights from the oracle's own generator), a 128-id prompt and
    8 greedy steps of one sequence; the per-token cost of the 2 layers is scaled to 24 and the
    head's cost added once. Returns (tokens/s, description)."""
    import dataclasses

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    from hwnpu_b200 import synth

    t0 = time.perf_counter()
    c3 = dataclasses.replace(synth.C3, name="c3-2layers", layers=2)
    model = synth.Model(c3, seed=0, gen=O.OracleGen)
    sess = O.OracleSession(model, 160, threads=threads)
    logits = sess.step(list(O.OracleGen.tokens(1, c3.vocab, 128)))[0]
    a = time.perf_counter()
    steps = 8
    for _ in range(steps):
        tok = O.lib().or_argmax_f16(O.p(logits, O._u16p), c3.vocab)
        logits = sess.step([tok])[0]
    per2 = (time.perf_counter() - a) / steps
    sess.close()
    # the head (201088 x 2880 bf16) is part of per2 once; the 2 layers are scaled to 24
    head_s = 201088 * 2880 * 2 / 20e9  # its bytes at a 20 GB/s host stream, a generous estimate
    per_tok = max(per2 - head_s, 0.0) * 12 + head_s
    wall = time.perf_counter() - t0
    return 1.0 / per_tok, (f"oracle C3 on {threads} threads: 2 of its 24 layers (full vocabulary) timed over "
                           f"{steps} greedy steps after a 128-id prompt, {1e3 * per2:.0f} ms a token, the layers "
                           f"scaled to 24 (batch 16 costs 16 tokens on the CPU); {wall:.0f} s of CPU work")


def run_reference(args, rank, world):
    """--impl reference: the oracle's C5 rate (and bs1 rate) on the host's cores, rank 0 only."""
    if rank != 0:
        return
    from hwnpu_b200 import _abi as A

    cores, model_name = cpu_info()
    if args.workload in ("default", "c5"):
        s = CpuSample(cores, A.HC_KV_INT8_PAGED)
        value = cpu_c5(s, world, args.steps)
        sample = s.describe() + f"; extrapolated to {args.steps} steps of the C5 schedule ({C5_SEQS} sequences)"
        config = c5_config(args, world)
    elif args.workload == "c3":
        value, sample = cpu_c3(cores)
        config = {"workload": f"C3 greedy decode after {C3_PROMPT}-id prompts, batch 16 (oracle sample)",
                  "model": "C3 24L d2880 64q/8kv hd64, 32 MXFP4 experts (2880) top-4, window 128, sinks, YaRN"}
    else:
        s = CpuSample(cores, A.HC_KV_F16)
        value = 1.0 / s.token_s(PROMPT + (PASS + 1) / 2.0)
        sample = s.describe() + f"; at the bs1 context {PROMPT}-{PROMPT + PASS}"
        config = bs1_config(args, world)
    base = {"value": value, "unit": "tokens/s", "cores": cores, "cpu": model_name, "kind": "port", "sample": sample}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "data": "synthetic",
            "config": config, "cpu_baseline": base,
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- the GPU side ---------------------------------------------------------------------------------
def c5_config(args, world):
    return {"workload": "C5 continuous-batched ragged decode: 64 sequences, contexts U[128,8192] (seed 2), "
                        "128 steps owed each (staggered), finished ones replaced by 512-id prompts; "
                        "paged int8 KV (16-position pages)",
            "model": "C2 28L d2048 16q/8kv hd128 FFN6144 V151936 tied, int4 asym g32",
            "global_batch": C5_SEQS, "parallelism": f"sequence shards x{world} (replicated weights)",
            "l2": "inputs larger than L2 (1.1 GB of weights and ~15 GB of KV a step)"}


def bs1_config(args, world):
    return {"workload": f"C2 bs1 greedy decode: {PROMPT}-id random prompt, passes of {PASS} steps "
                        f"(context {PROMPT}-{PROMPT + PASS})",
            "model": "C2 28L d2048 16q/8kv hd128 FFN6144 V151936 tied, int4 asym g32",
            "global_batch": world, "seq_len": PROMPT + PASS, "prompt": PROMPT, "steps_per_pass": PASS,
            "parallelism": f"replicas x{world}", "l2": "inputs larger than L2 (the weights, ~1.1 GB, stream every token)"}


def source_sha(rel):
    try:
        return hashlib.sha1(open(os.path.join(ROOT, rel), "rb").read()).hexdigest()[:16]
    except OSError:
        return None


def profiled_traffic(name):
    """DRAM bytes a launch of the named kernel moved in an ncu capture (profiles/<name>.json), when
    the kernel's source file is still the one captured; else None."""
    try:
        rec = json.load(open(os.path.join(ROOT, "profiles", name + ".json")))
    except Exception:
        return None, None
    if rec.get("source_sha1") != source_sha(rec.get("source", "")):
        return None, f"profiles/{name}.json is from another build of {rec.get('source')}"
    return rec.get("dram_bytes_per_launch"), f"profiles/{name}.json ({rec.get('workload')})"


def kernel_roofline(dev, lin, ntok, label, profile_name, reps=50):
    """The GEMV class of a step on one of its matrices, timed alone: reps calls of hc_linear_run
    (its activation launch, if any, included) captured in one CUDA graph, as a step runs them, and
    timed with CUDA events around the graph's replay on torch's stream; algorithmic bytes = the
    matrix's weight bytes per call."""
    import ctypes as C

    import torch

    from hwnpu_b200 import _abi as A

    h = C.c_void_p()
    A.check(A.lib().hc_linear_load(dev.h, C.byref(lin.desc()), C.byref(h)))
    x = torch.randn(ntok, lin.cols, device="cuda")
    y = torch.empty(ntok, lin.rows, device="cuda")
    cs = torch.cuda.current_stream()

    def once(st):
        A.check(A.lib().hc_linear_run(h, C.c_void_p(x.data_ptr()), ntok, C.c_void_p(y.data_ptr()),
                                      C.c_void_p(st.cuda_stream)))

    for _ in range(5):
        once(cs)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gs = torch.cuda.current_stream()
        for _ in range(reps):
            once(gs)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    graph.replay()
    e1.record(cs)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del graph
    A.lib().hc_linear_free(h)
    wbytes = sum(a.nbytes for a in (lin.data, lin.scales, lin.zeros, lin.exps) if a is not None)
    peak, kind = peaks()
    ach = wbytes / (ms / 1e3) / 1e9
    traffic, source = profiled_traffic(profile_name)
    return {"bound": "hbm", "kernel": label, "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
            "peak_kind": kind, "traffic": traffic, "traffic_source": source, "bytes_per_launch": wbytes,
            "ms_per_launch": ms, "tokens": ntok}


def run_bs1(args, lm, model, dev, world, dist, K, W):
    """C2 bs1 on this rank: the device-resident loop (value) and the public per-token call (e2e)."""
    import torch

    from hwnpu_b200 import replicas, synth

    sess = lm.session(max_context=PROMPT + PASS + W + 8, max_step=8)
    prompt = synth.tokens(1, model.cfg.vocab, PROMPT)
    first = sess.greedy(prompt)
    base = sess.pos()
    sess.generate(first, W)
    sess.truncate(base)
    stream = torch.cuda.ExternalStream(sess.stream())
    if args.profile:  # --profile N: N greedy steps between cudaProfilerStart/Stop (for ncu), no timing
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        sess.generate(first, args.profile)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        sess.close()
        return None
    launches0 = sess.stats()["launches"]

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    done = 0
    while done < K:
        n = min(PASS, K - done)
        sess.generate(first, n)
        sess.truncate(base)
        done += n
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    launches = sess.stats()["launches"] - launches0
    barrier()
    E = min(K, PASS)
    tok = first
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(E):
        tok = sess.greedy([tok])
    f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    sess.truncate(base)
    sess.close()
    barrier()
    t_max = replicas.job_time(ms, dist, "cuda")
    t_e2e = replicas.job_time(ms_e2e, dist, "cuda")
    cfg = model.cfg
    kv_per_pos = cfg.layers * cfg.kv_heads * cfg.head_dim * 2 * 2
    bytes_tok = lm.weight_bytes + kv_per_pos * (PROMPT + (PASS + 1) / 2.0)
    peak, peak_kind = peaks()
    per_gpu = K / (t_max / 1e3)
    return {"value": world * K / (t_max / 1e3), "unit": "tokens/s", "ms_per_step": t_max / K, "steps": K,
            "e2e": {"value": world * E / (t_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 4 * world,
                    "d2h_bytes_per_step": 4 * world, "api": "hc_step per token (token in, greedy choice out)"},
            "gpu_launches": int(launches), "path": "kernel sequence (CUDA graph, PDL-chained)",
            "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs": bytes_tok * per_gpu / 1e9,
                              "frac": bytes_tok * per_gpu / 1e9 / peak, "peak": peak, "peak_kind": peak_kind,
                              "ideal_tokens_per_s": peak * 1e9 / bytes_tok},
            "config": bs1_config(args, world)}


def run_c5(args, lm, world, rank, dist, K, W):
    """The C5 batch of this rank (see the module docstring); returns the line's C5 figures."""
    import torch

    from hwnpu_b200 import _abi as A
    from hwnpu_b200 import replicas, synth

    mine = replicas.shard(C5_SEQS, rank, world)
    n = len(mine)
    ctx_all = c5_contexts()
    max_ctx = int(ctx_all.max()) + C5_OWED + W + K + 16
    warm = n  # an extra slot that runs the chunk shapes once before the timed steps
    sess = lm.session(max_context=max_ctx, max_seqs=n + 1, kv_format=A.HC_KV_INT8_PAGED)
    for k in range(1, 9):
        sess.step_batch([warm], [synth.tokens(7, synth.C2.vocab, k)], want_logits=False)
    sess.reset(warm)
    sch = C5Schedule(mine)
    t_fill = time.perf_counter()
    last = []
    for i, g in enumerate(mine):
        _, am = sess.step_batch([i], [synth.tokens(100 + g, synth.C2.vocab, int(ctx_all[g]))], want_logits=False)
        last.append(int(am[0]))
    torch.cuda.synchronize()
    fill_s = time.perf_counter() - t_fill
    stream = torch.cuda.ExternalStream(sess.stream())

    def run(steps, timed):
        dec = prm = 0
        dev_ms = kv = 0.0
        for _ in range(steps):
            plan = sch.step()
            lists = []
            for i, (kind, seed) in enumerate(plan):
                if kind == "prompt":
                    sess.reset(i)
                    lists.append(synth.tokens(seed, synth.C2.vocab, C5_NEW_PROMPT))
                else:
                    lists.append([last[i]])
            pos0 = [sess.pos(i) for i in range(n)] if timed else None
            _, am = sess.step_batch(list(range(n)), lists, want_logits=False)
            for i in range(n):
                last[i] = int(am[i])
            dec += n
            prm += sum(len(l) - 1 for l in lists)
            if timed:
                dev_ms += sess.stats()["last_step_us"] / 1e3
                for i in range(n):  # KV positions each token attends to (its own row included)
                    m = len(lists[i])
                    kv += C5_KV_POS * (m * pos0[i] + m * (m + 1) / 2)
        return dec, prm, dev_ms, kv

    run(W, False)
    if args.profile:  # --profile N: N more steps between cudaProfilerStart/Stop (for ncu), no timing
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        run(args.profile, False)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        sess.close()
        return None
    launches0 = sess.stats()["launches"]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dec, prm, dev_ms, kv = run(K, True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    launches = sess.stats()["launches"] - launches0
    sess.close()
    t_dev = replicas.job_time(dev_ms, dist, "cuda")
    t_e2e = replicas.job_time(e2e_ms, dist, "cuda")
    dec_all = replicas.job_total(dec, dist, "cuda")
    prm_all = replicas.job_total(prm, dist, "cuda")
    kv_all = replicas.job_total(int(kv), dist, "cuda")
    peak, peak_kind = peaks()
    step_bytes = world * K * lm.weight_bytes + kv_all  # each rank reads its weights once a step
    ach = step_bytes / (t_dev / 1e3) / 1e9 / world
    return {"value": dec_all / (t_dev / 1e3), "ms_per_step": t_dev / K, "decoded_tokens": dec_all,
            "prompt_tokens_read": prm_all, "prompt_tokens_per_s": prm_all / (t_dev / 1e3),
            "e2e": {"value": dec_all / (t_e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * (dec_all + prm_all) // K + 12 * C5_SEQS,
                    "d2h_bytes_per_step": 4 * C5_SEQS,
                    "api": "hc_step over every slot a step (host-built token lists in, greedy choices out)"},
            "gpu_launches": int(launches),
            "step_roofline": {"bytes_per_step": step_bytes / K, "achieved_gbs_per_gpu": ach, "peak": peak,
                              "peak_kind": peak_kind, "frac": ach / peak,
                              "weights_bytes_per_rank_step": lm.weight_bytes, "kv_bytes_per_step": kv_all / K},
            "fill": {"slots_rank0": n, "seconds_rank0": fill_s}}


def run_default(args, rank, world, local, dist):
    import torch

    import hwnpu_b200 as hb

    K, W = args.steps, max(3, args.warmup)
    dev = hb.Device(local)
    if args.layers and not args.profile:
        raise SystemExit("--layers only shrinks the model of a --profile capture; bench lines use all 28")
    cfg = dataclasses.replace(hb.C2, layers=args.layers) if args.layers else hb.C2
    model = hb.Model(cfg, seed=0)
    lm = dev.load_model(model)
    clocks = Clocks(local)
    clocks.start()
    c5 = run_c5(args, lm, world, rank, dist, K, W)
    clk = clocks.stop()
    if c5 is None:
        return
    bs1 = run_bs1(args, lm, model, dev, world, dist, K, W)
    # the GEMV class of the C5 step (its chunks of 64 tokens), on the largest matrix of a layer
    # (gate/up, 12288 x 2048): the tensor-core GEMV (tcgen05, tokens on the MMA's N)
    gu = hb.synth.Linear.quantize(hb.synth.normal(5, "bench.gate_up", 12288 * 2048, 0.02).reshape(12288, 2048),
                                  hb._abi.HC_FMT_INT4_ASYM_G32)
    roof = kernel_roofline(dev, gu, 64, "tc_gemm_kernel<int4> (tcgen05.mma, 64 tokens) on the C2 gate/up "
                           "12288x2048 (+ its fp16 operand writer)", "tc_gemm_c2_gateup64")
    bs1["roofline"] = kernel_roofline(dev, gu, 1, "gemv_kernel<int4, 1 token> on the C2 gate/up 12288x2048 "
                                      "(its activation quantisation built in)", "gemv_c2_gateup1")
    lm.close()
    dev.close()
    if dist:
        dist.barrier()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": c5["value"], "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": c5["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights x int8 (hi+lo) activations -> int32, f32 scaling; int8 KV x fp16 page scales",
            "data": "synthetic (seeded N(0,0.02) weights, uniform ids)", "config": c5_config(args, world),
            "e2e": c5["e2e"], "gpu_launches": c5["gpu_launches"], "roofline": roof,
            "step_roofline": c5["step_roofline"], "decoded_tokens": c5["decoded_tokens"],
            "prompt_tokens_read": c5["prompt_tokens_read"], "prompt_tokens_per_s": c5["prompt_tokens_per_s"],
            "fill": c5["fill"], "clocks": clk, "bs1": bs1}
    if world == 1 and not args.no_cpu_baseline:
        try:
            from hwnpu_b200 import _abi as A

            cores, cpu_model = cpu_info()
            s = CpuSample(cores, A.HC_KV_INT8_PAGED)
            v = cpu_c5(s, world, K)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "cpu": cpu_model, "kind": "port",
                                    "sample": s.describe() + f"; extrapolated to the {K} timed steps of the C5 schedule"}
            s16 = CpuSample(cores, A.HC_KV_F16)
            bs1["cpu_baseline"] = {"value": 1.0 / s16.token_s(PROMPT + (PASS + 1) / 2.0), "unit": "tokens/s",
                                   "cores": cores, "cpu": cpu_model, "kind": "port", "sample": s16.describe()}
        except Exception as e:  # the baseline is reported, not required for the GPU number
            line["cpu_baseline"] = {"value": None, "error": str(e)[:300]}
    print(json.dumps(line), flush=True)


def run_bs1_line(args, rank, world, local, dist, workload):
    """--workload c2 / c1: the bs1 line alone (weak scaling: a sequence a rank)."""
    import hwnpu_b200 as hb

    K, W = args.steps, max(3, args.warmup)
    dev = hb.Device(local)
    model = hb.Model({"c2": hb.C2, "c1": hb.C1}[workload], seed=0)
    lm = dev.load_model(model)
    clocks = Clocks(local)
    clocks.start()
    r = run_bs1(args, lm, model, dev, world, dist, K, W)
    clk = clocks.stop()
    lm.close()
    dev.close()
    if rank != 0 or r is None:
        return
    cfg = r.pop("config")
    if workload == "c1":
        cfg["workload"] = cfg["workload"].replace("C2", "C1")
        cfg["model"] = "C1 4L d1024 16q/4kv hd64 FFN2816 V32000, int8 rows"
    line = {"metric": "decode tokens/s", "unit": "tokens/s", "n_gpus": world, "warmup": W, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4/int8 weights x int8 (hi+lo) activations",
            "data": "synthetic (seeded N(0,0.02) weights, uniform ids)", "config": cfg, "clocks": clk, **r}
    print(json.dumps(line), flush=True)


C3_PROMPT = 2048


def run_c3(args, rank, world, local, dist):
    """C3: the gpt-oss-shaped MoE model (24 layers, 32 MXFP4 experts of
    2880, top 4, bf16 attention with sinks and 128-token windows on alternate layers), greedy decode
    after 2048-id prompts at batch 1 (value: the device-resident loop, hc_generate) and batch 16 (16
    sequences stepped together by hc_step, their experts grouped over the 16 tokens). One replica a
    GPU. Weights: seeded synthetic tensors of the architecture (router N(0, 1/hidden) so that its
    logits are about N(0, 1))."""
    import torch

    import hwnpu_b200 as hb
    from hwnpu_b200 import replicas, synth

    K, W = min(args.steps, 256), max(3, args.warmup)
    torch.cuda.set_device(local)
    dev = hb.Device(local)
    t0 = time.perf_counter()
    model = hb.Model(hb.C3, seed=0)
    build_s = time.perf_counter() - t0
    lm = dev.load_model(model)
    load_s = time.perf_counter() - t0 - build_s
    cfg = model.cfg
    ctx = C3_PROMPT + K + W + 8
    clocks = Clocks(local)
    clocks.start()

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    # batch 1: device-resident loop (value) and the per-token public call (e2e)
    s1 = lm.session(max_context=ctx, max_step=8)
    first = s1.greedy(synth.tokens(1, cfg.vocab, C3_PROMPT))
    base = s1.pos()
    s1.generate(first, W)
    s1.truncate(base)
    st1 = torch.cuda.ExternalStream(s1.stream())
    l0 = s1.stats()["launches"]
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st1)
    s1.generate(first, K)
    e1.record(st1)
    torch.cuda.synchronize()
    ms1 = e0.elapsed_time(e1)
    launches1 = s1.stats()["launches"] - l0
    s1.truncate(base)
    E = min(K, 64)
    tok = first
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(st1)
    for _ in range(E):
        tok = s1.greedy([tok])
    f1.record(st1)
    torch.cuda.synchronize()
    ms1_e2e = f0.elapsed_time(f1)
    s1.close()

    # batch 16: every sequence's next token in one hc_step a step
    B = 16
    s16 = lm.session(max_context=ctx, max_seqs=B, max_step=8)
    last = []
    t_fill = time.perf_counter()
    for i in range(B):
        _, am = s16.step_batch([i], [synth.tokens(10 + i, cfg.vocab, C3_PROMPT)], want_logits=False)
        last.append(int(am[0]))
    torch.cuda.synchronize()
    fill_s = time.perf_counter() - t_fill
    st16 = torch.cuda.ExternalStream(s16.stream())

    def run(steps):
        dev_ms = 0.0
        for _ in range(steps):
            _, am = s16.step_batch(list(range(B)), [[t] for t in last], want_logits=False)
            last[:] = [int(a) for a in am]
            dev_ms += s16.stats()["last_step_us"] / 1e3
        return dev_ms

    run(W)
    l0 = s16.stats()["launches"]
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(st16)
    dev16 = run(K)
    g1.record(st16)
    torch.cuda.synchronize()
    ms16_e2e = g0.elapsed_time(g1)
    launches16 = s16.stats()["launches"] - l0
    s16.close()
    clk = clocks.stop()
    barrier()
    t1 = replicas.job_time(ms1, dist, "cuda")
    t1e = replicas.job_time(ms1_e2e, dist, "cuda")
    t16 = replicas.job_time(dev16, dist, "cuda")
    t16e = replicas.job_time(ms16_e2e, dist, "cuda")
    peak, peak_kind = peaks()
    # bytes a token reads at batch 1: the attention, router and head weights, top_k experts (the
    # model's weight_bytes), and the cache its layers attend to (windowed layers 128 positions)
    kv_pos = cfg.kv_heads * cfg.head_dim * 2 * 2
    mid = C3_PROMPT + K / 2.0
    kv_tok = kv_pos * (cfg.layers // 2) * (mid + min(mid, cfg.window))
    b1 = lm.weight_bytes + kv_tok
    per1 = K / (t1 / 1e3)
    lm.close()
    dev.close()
    if rank != 0:
        return
    line = {"metric": "decode tokens/s (C3 MoE, batch 16; batch 1 nested)", "value": world * B * K / (t16 / 1e3),
            "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": t16 / K,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "MXFP4 experts x int8 activations (integer block sums); bf16 attention/router/head x f32",
            "data": "synthetic (seeded weights of the architecture, uniform ids)",
            "config": {"workload": f"C3 greedy decode after {C3_PROMPT}-id prompts, batch 16 (16 sequences a "
                                   f"replica), {K} steps", "model": "C3 24L d2880 64q/8kv hd64, 32 MXFP4 experts "
                                   "(2880) top-4, window 128 on even layers, sinks, YaRN, V201088",
                       "global_batch": world * B, "seq_len": ctx, "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (the attention and head weights, ~2.4 GB, stream every step)"},
            "e2e": {"value": world * B * K / (t16e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 4 * B * 3,
                    "d2h_bytes_per_step": 4 * B, "api": "hc_step over the 16 sequences a step"},
            "gpu_launches": int(launches16), "clocks": clk, "model_build_s": build_s, "model_load_s": load_s,
            "fill": {"sequences": B, "seconds": fill_s},
            "bs1": {"value": world * K / (t1 / 1e3), "unit": "tokens/s", "ms_per_step": t1 / K,
                    "e2e": {"value": world * E / (t1e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                            "d2h_bytes_per_step": 4, "api": "hc_step per token"},
                    "gpu_launches": int(launches1),
                    "step_roofline": {"bytes_per_token": b1, "achieved_gbs": b1 * per1 / 1e9,
                                      "frac": b1 * per1 / 1e9 / peak, "peak": peak, "peak_kind": peak_kind}}}
    print(json.dumps(line), flush=True)


def run_c4(args, rank, world, local, dist):
    """C4: greedy speculative decoding, the C1-shaped int8 draft (vocab
    151936) drafting k = 4 tokens a round and the C2 target verifying the 5 rows in one hc_speculate
    call with greedy acceptance (chat/engine.go:1044-1058); 512 tokens from a 512-id prompt. The
    output must equal plain greedy decoding of the target, which is checked here. One replica a
    GPU; the whole-job tokens/s sums the replicas over the slowest one's time."""
    import numpy as np
    import torch

    import hwnpu_b200 as hb
    from hwnpu_b200 import synth

    P, OUT, k = 512, 512, 4
    dev = hb.Device(local)
    lt = dev.load_model(hb.Model(hb.C2, seed=0))
    ld = dev.load_model(hb.Model(hb.C4_DRAFT, seed=1))
    ctx = P + OUT + 2 * k + 8
    prompt = synth.tokens(3, hb.C2.vocab, P)

    # plain greedy decoding of the target: the stream speculation must reproduce, and its speed
    plain = lt.session(max_context=ctx)
    first = plain.greedy(prompt)
    base = plain.pos()
    plain.generate(first, 8)
    plain.truncate(base)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ref = [first] + [int(x) for x in plain.generate(first, OUT - 1)]
    plain_s = time.perf_counter() - t0
    plain.close()

    def speculate_run():
        ts = lt.session(max_context=ctx, max_step=k + 1)
        ds = ld.session(max_context=ctx)
        out = [ts.greedy(prompt)]
        ds.greedy(prompt)
        pending, rounds, accepted = [], 0, 0
        while len(out) < OUT:
            last = out[-1]
            if pending:
                ds.greedy(pending)  # an accepted draft the draft model has not read yet
            d = [int(x) for x in ds.generate(last, k)]  # reads last, d1..d3; d4 is only written
            kept, nxt, _ = ts.speculate_tokens([last] + d)
            acc = kept - 1
            out.extend(d[:acc])
            out.append(nxt)
            p_last = ds.pos() - k  # the draft cache's position of `last`
            if acc < k:
                ds.truncate(p_last + 1 + acc)
                pending = []
            else:
                pending = [d[k - 1]]
            rounds += 1
            accepted += acc
        ts.close()
        ds.close()
        return out[:OUT], rounds, accepted

    speculate_run()  # warm-up (graphs of every shape)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out, rounds, accepted = speculate_run()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    from hwnpu_b200 import replicas

    t_max = replicas.job_time(dt, dist, "cuda")
    same = out == ref[:OUT]
    if rank != 0:
        return
    round_bytes = 4 * (45.2e6 + 155.6e6) + 1.0755e9 + 5 * 112 * 1024 * (P + OUT / 2)
    line = {"metric": "speculative decode tokens/s", "value": world * OUT / t_max, "unit": "tokens/s",
            "n_gpus": world, "steps": rounds, "warmup": 1, "ms_per_step": 1e3 * t_max / rounds,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8/int4 x int8(hi+lo) MMA -> int32, f32 scaling",
            "data": "synthetic (seeded N(0,0.02) weights; draft and target independent, so drafts rarely match)",
            "config": {"workload": "C4 speculative decode: C1-shaped int8 draft (V151936) -> C2 target, k=4, "
                                   "512 tokens from a 512-id prompt, bs1", "global_batch": world,
                       "parallelism": f"replicas x{world}", "k": k, "prompt": P, "tokens": OUT},
            "rounds": rounds, "accepted_per_round": accepted / rounds,
            "tokens_per_round": OUT / rounds, "identical_to_greedy": same,
            "plain_greedy_tokens_per_s": OUT / plain_s,
            "e2e": {"value": world * OUT / t_max, "unit": "tokens/s", "h2d_bytes_per_step": 4 * (k + 1) + 4 * k,
                    "d2h_bytes_per_step": 4 * k + 8,
                    "api": "hc_generate (draft) + hc_speculate (target verify) per round, host-driven"},
            "round_bytes_model": round_bytes}
    print(json.dumps(line), flush=True)
    if not same:
        raise SystemExit("speculative output differs from plain greedy decoding")



def run_linear(args, local):
    """One C2-shaped matrix (hc_linear_load) run over --ntok tokens (hc_linear_run), timed with CUDA
    events on torch's stream: the GEMV kernels alone, for tuning and for ncu on a small case."""
    import ctypes as C

    import torch

    import hwnpu_b200 as hb
    from hwnpu_b200 import _abi as A
    from hwnpu_b200 import synth

    torch.cuda.set_device(local)
    dev = hb.Device(local)
    rows, cols, n = args.rows, args.cols, args.ntok
    w = synth.normal(5, f"lin{rows}x{cols}", rows * cols, 0.02).reshape(rows, cols)
    lin = synth.Linear.quantize(w, A.HC_FMT_INT4_ASYM_G32)
    h = C.c_void_p()
    A.check(A.lib().hc_linear_load(dev.h, C.byref(lin.desc()), C.byref(h)))
    x = torch.randn(n, cols, device="cuda")
    y = torch.empty(n, rows, device="cuda")
    cs = torch.cuda.current_stream()

    def once():
        A.check(A.lib().hc_linear_run(h, C.c_void_p(x.data_ptr()), n, C.c_void_p(y.data_ptr()), C.c_void_p(cs.cuda_stream)))

    for _ in range(max(3, args.warmup)):
        once()
    if args.profile:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for _ in range(args.profile):
            once()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    reps = max(1, args.steps)
    # the reps calls as one CUDA graph (as a step runs them), timed around its replay
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gs = torch.cuda.current_stream()
        for _ in range(reps):
            A.check(A.lib().hc_linear_run(h, C.c_void_p(x.data_ptr()), n, C.c_void_p(y.data_ptr()),
                                          C.c_void_p(gs.cuda_stream)))
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    graph.replay()
    e1.record(cs)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del graph
    wbytes = lin.data.nbytes + lin.scales.nbytes + (lin.zeros.nbytes if lin.zeros is not None else 0)
    peak, kind = peaks()
    print(json.dumps({"workload": "linear", "rows": rows, "cols": cols, "ntok": n, "us_per_call": ms * 1e3,
                      "weight_gbs": wbytes / (ms / 1e3) / 1e9, "frac_hbm": wbytes / (ms / 1e3) / 1e9 / peak,
                      "int_tops_useful": 2.0 * rows * cols * n / (ms / 1e3) / 1e12,
                      "note": "a CUDA graph of the calls; includes the activation quantiser launch, if any"}), flush=True)
    A.lib().hc_linear_free(h)
    dev.close()




def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["default", "c5", "c2", "c1", "c3", "c4", "linear"], default="default",
                    help="default: the C5 64-sequence ragged decode line with the C2 bs1 figures nested; "
                         "c2 / c1: a bs1 line alone; c3: the gpt-oss-shaped MoE at batch 1 and 16; c4: speculative decoding (C1-shaped int8 draft with V151936 "
                         "-> C2 target, k=4, 512 tokens from a 512-id prompt); linear: one GEMV")
    ap.add_argument("--rows", type=int, default=12288, help="--workload linear: matrix rows")
    ap.add_argument("--cols", type=int, default=2048, help="--workload linear: matrix columns")
    ap.add_argument("--ntok", type=int, default=64, help="--workload linear: tokens a call")
    ap.add_argument("--profile", type=int, default=0,
                    help="--workload linear / c5: run this many calls (steps) between cudaProfilerStart/Stop "
                         "after the warm-up, for ncu (c5: then exit without timing)")
    ap.add_argument("--layers", type=int, default=0,
                    help="with --profile on the C5 workload: a model of this many C2 layers (a small ncu case)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "linear":
        run_linear(args, local)
        return

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    if args.workload in ("default", "c5"):
        run_default(args, rank, world, local, dist)
    elif args.workload == "c4":
        run_c4(args, rank, world, local, dist)
    elif args.workload == "c3":
        run_c3(args, rank, world, local, dist)
    else:
        run_bs1_line(args, rank, world, local, dist, args.workload)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
