#!/usr/bin/env python
"""Decode benchmark of the B200 engine on BASELINE configs[1] (C2): a 28-layer 1.7B Qwen3
decoder with int4 asymmetric group-32 weights, batch 1, a 1024-id random prompt, greedy steps.

A step is one decoded token. The timed region runs K tokens as passes of 256 greedy steps from
the same 1024-token prompt (the KV cache is truncated back to the prompt after each pass, so the
context stays in 1024..1280, the configuration's). value: tokens/s of the device-resident loop
(hc_generate: tokens fed back on the device), timed with CUDA events on the session's stream.
e2e: the same through the per-token public call hc_step (token H2D, greedy choice D2H each step).

Under torchrun (N > 1) every rank runs its own replica (sequences are independent; weights are
replicated; no collective on the path): value = all ranks' tokens / the slowest rank's time.

--impl reference times the reference path's CPU restatement (oracle/, the Go path cannot run
here) on the host's cores for the same metric, rank 0 only.
"""

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT = 1024
PASS = 256


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region (clock and throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.p, self.path = gpu, None, None

    def start(self):
        try:
            os.makedirs(os.path.join(ROOT, "gpurun_out"), exist_ok=True)
            self.path = os.path.join(ROOT, "gpurun_out", f"clocks_{self.gpu}_{os.getpid()}.csv")
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-i", str(self.gpu), "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_model(workload):
    import hwnpu_b200 as hb

    cfg = {"c2": hb.C2, "c1": hb.C1}[workload]
    return hb.Model(cfg, seed=0)


def cpu_generate(model, prompt_len, steps, threads):
    """The oracle (the reference path restated on the CPU): tokens/s of greedy decode steps after
    a prefilled prompt; returns (tokens/s, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import numpy as np
    import oracle_lib as O
    from hwnpu_b200 import synth

    s = O.OracleSession(model, prompt_len + steps + 1, threads=threads)
    toks = synth.tokens(1, model.cfg.vocab, prompt_len)
    logits = s.step(toks)[0]
    t0 = time.perf_counter()
    for _ in range(steps):
        t = O.lib().or_argmax_f16(O.p(logits, O._u16p), model.cfg.vocab)
        logits = s.step([t])[0]
    dt = time.perf_counter() - t0
    s.close()
    return steps / dt, dt


def run_reference(args, rank):
    if rank != 0:
        return
    model = build_model(args.workload)
    threads = os.cpu_count()
    steps = max(1, min(args.steps, 16))
    tps, dt = cpu_generate(model, 64, steps, threads)
    sample = (f"{steps} greedy decode tokens of the {args.workload.upper()} model after a 64-id prompt "
              f"(per-token cost is the fp32 weight stream: the KV of 1024-1280 positions is ~2% of it)")
    line = {"impl": "reference", "metric": "decode tokens/s", "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": 0, "higher_is_better": True, "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
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


C5_SEQS, C5_STEPS, C5_NEW_PROMPT = 64, 128, 512
C5_KV_POS = 28 * (8 * 128 * 2 + 2 * 8 * 2 / 16)  # int8 K and V rows + fp16 page scales, per position


def run_c5(args, rank, world, local, dist):
    """C5: continuous-batched ragged decode of the C2 model over a paged
    int8 KV cache (16-position pages, fp16 scale per page and KV head). 64 sequences with contexts
    drawn uniform on 128..8192 (PCG64, seed 2), each owed 128 decode steps; the owed counts are
    staggered (sequence i has 128 - 2i left) so that sequences finish at different steps, and a
    finished one is replaced in its slot by a new sequence whose 512-id prompt is read in the same
    batched step as the others' decode tokens. The 64 sequences are sharded round robin over the
    ranks (replicas.shard), weights replicated, no collective on the path.

    A timed step is one hc_step call over every slot of the rank (each slot's next token, or a new
    prompt). value: the decoded tokens of all ranks / the slowest rank's device time (the sum of the
    call's chunk graphs, CUDA events). e2e: the same tokens over CUDA events around the whole host
    loop (token lists in, greedy choices out, slot replacement), max over ranks."""
    import numpy as np
    import torch

    import hwnpu_b200 as hb
    from hwnpu_b200 import _abi as A
    from hwnpu_b200 import replicas, synth

    ctx_all = np.random.default_rng(2).integers(128, 8192, size=C5_SEQS, endpoint=True)
    mine = replicas.shard(C5_SEQS, rank, world)
    n = len(mine)
    dev = hb.Device(local)
    model = hb.Model(hb.C2, seed=0)
    lm = dev.load_model(model)
    max_ctx = int(ctx_all.max()) + C5_STEPS + 16
    warm = n  # an extra slot that runs the chunk shapes once before the timed steps
    sess = lm.session(max_context=max_ctx, max_seqs=n + 1, kv_format=A.HC_KV_INT8_PAGED)
    for k in range(1, 9):
        sess.step_batch([warm], [synth.tokens(7, hb.C2.vocab, k)], want_logits=False)
    sess.reset(warm)

    # the starting state: every slot's context read as a prompt (untimed)
    t_fill = time.perf_counter()
    last, owed, ctx_tok = [], [], 0
    for i, gi in enumerate(mine):
        _, am = sess.step_batch([i], [synth.tokens(100 + gi, hb.C2.vocab, int(ctx_all[gi]))], want_logits=False)
        last.append(int(am[0]))
        owed.append(C5_STEPS - 2 * gi)
        ctx_tok += int(ctx_all[gi])
    torch.cuda.synchronize()
    fill_s = time.perf_counter() - t_fill
    stream = torch.cuda.ExternalStream(sess.stream())
    new_seed = [1000 + gi * 64 for gi in mine]

    def run(steps, timed):
        """`steps` batched steps; returns (decoded tokens, prompt tokens, device ms, kv bytes)."""
        dec = prm = 0
        dev_ms = kv = 0.0
        for _ in range(steps):
            lists, fresh = [], []
            for i in range(n):
                if owed[i] <= 0:  # finished: a new sequence takes the slot
                    sess.reset(i)
                    new_seed[i] += 1
                    lists.append(synth.tokens(new_seed[i], hb.C2.vocab, C5_NEW_PROMPT))
                    owed[i] = C5_STEPS
                    fresh.append(i)
                else:
                    lists.append([last[i]])
            pos0 = [sess.pos(i) for i in range(n)] if timed else None
            _, am = sess.step_batch(list(range(n)), lists, want_logits=False)
            for i in range(n):
                last[i] = int(am[i])
                owed[i] -= 1
            dec += n
            prm += sum(len(l) - 1 for l in lists)
            if timed:
                dev_ms += sess.stats()["last_step_us"] / 1e3
                for i in range(n):  # KV positions each token attends to (its own row included)
                    m = len(lists[i])
                    kv += C5_KV_POS * (m * pos0[i] + m * (m + 1) / 2)
        return dec, prm, dev_ms, kv

    W = max(3, args.warmup)
    run(W, False)
    if args.profile:  # a few steps between cudaProfilerStart/Stop (for ncu --profile-from-start off)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        dec, prm, dev_ms, _ = run(args.profile, True)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"profiled_steps": args.profile, "decoded": dec, "prompt_tokens": prm,
                          "device_ms": dev_ms}), flush=True)
        sess.close()
        lm.close()
        dev.close()
        return
    launches0 = sess.stats()["launches"]
    clocks = Clocks(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dec, prm, dev_ms, kv = run(C5_STEPS, True)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    e2e_ms = e0.elapsed_time(e1)
    launches = sess.stats()["launches"] - launches0
    t_dev = replicas.job_time(dev_ms, dist, "cuda")
    t_e2e = replicas.job_time(e2e_ms, dist, "cuda")
    dec_all = replicas.job_total(dec, dist, "cuda")
    prm_all = replicas.job_total(prm, dist, "cuda")
    kv_all = replicas.job_total(int(kv), dist, "cuda")
    weight_bytes = lm.weight_bytes
    sess.close()
    lm.close()
    dev.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = peaks()
    # algorithmic bytes: each rank reads its weights once per step, plus the KV every token touches
    step_bytes = world * C5_STEPS * weight_bytes + kv_all
    ach = step_bytes / (t_dev / 1e3) / 1e9 / world  # per GPU
    line = {
        "metric": "decode tokens/s", "value": dec_all / (t_dev / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": C5_STEPS, "warmup": W, "ms_per_step": t_dev / C5_STEPS, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 x int8(hi+lo) MMA -> int32, f32 scaling; int8 KV x fp16 page scales",
        "data": "synthetic (seeded N(0,0.02) weights, uniform ids)",
        "config": {"workload": "C5 continuous-batched ragged decode: 64 sequences, contexts U[128,8192] (seed 2), "
                               "128 steps owed each (staggered), finished ones replaced by 512-id prompts; "
                               "paged int8 KV (16-position pages)",
                   "model": "C2 28L d2048 16q/8kv hd128 FFN6144 V151936 tied, int4 asym g32",
                   "global_batch": C5_SEQS, "parallelism": f"sequence shards x{world} (replicated weights)",
                   "l2": "inputs larger than L2 (1.1 GB of weights and ~15 GB of KV a step)"},
        "decoded_tokens": dec_all, "prompt_tokens_read": prm_all,
        "prompt_tokens_per_s": prm_all / (t_dev / 1e3),
        "e2e": {"value": dec_all / (t_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 16 * (dec_all + prm_all) // C5_STEPS,
                "d2h_bytes_per_step": 4 * dec_all // C5_STEPS,
                "api": "hc_step over every slot per step (host-built token lists, greedy choices out)"},
        "gpu_launches": int(launches),
        "step_roofline": {"bytes_per_step": step_bytes / C5_STEPS, "achieved_gbs_per_gpu": ach, "peak": peak,
                          "peak_kind": peak_kind, "frac": ach / peak,
                          "weights_bytes_per_rank_step": weight_bytes, "kv_bytes_per_step": kv_all / C5_STEPS},
        "fill": {"context_tokens_rank0": ctx_tok, "seconds_rank0": fill_s},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


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
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    for _ in range(reps):
        once()
    e1.record(cs)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    wbytes = lin.data.nbytes + lin.scales.nbytes + (lin.zeros.nbytes if lin.zeros is not None else 0)
    peak, kind = peaks()
    print(json.dumps({"workload": "linear", "rows": rows, "cols": cols, "ntok": n, "us_per_call": ms * 1e3,
                      "weight_gbs": wbytes / (ms / 1e3) / 1e9, "frac_hbm": wbytes / (ms / 1e3) / 1e9 / peak,
                      "int_tops_useful": 2.0 * rows * cols * n / (ms / 1e3) / 1e12,
                      "note": "includes the activation quantiser launch(es)"}), flush=True)
    A.lib().hc_linear_free(h)
    dev.close()


def workload_config(args):
    return {"workload": f"{args.workload.upper()} bs1 greedy decode: 1024-id random prompt, passes of 256 steps "
                        f"(context 1024-1280)",
            "model": "C2 28L d2048 16q/8kv hd128 FFN6144 V151936 tied, int4 asym g32" if args.workload == "c2"
            else "C1 4L d1024 16q/4kv hd64 FFN2816 V32000, int8 rows",
            "global_batch": args.gpus, "seq_len": PROMPT + PASS, "prompt": PROMPT, "steps_per_pass": PASS,
            "parallelism": f"replicas x{args.gpus}", "l2": "inputs larger than L2 (the weights, ~1.1 GB, stream every token)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2560)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=12288, help="--workload linear: matrix rows")
    ap.add_argument("--cols", type=int, default=2048, help="--workload linear: matrix columns")
    ap.add_argument("--ntok", type=int, default=64, help="--workload linear: tokens a call")
    ap.add_argument("--workload", choices=["c2", "c1", "c4", "c5", "linear"], default="c2",
                    help="c2: the headline bs1 decode; c1: the small int8 model; c4: speculative decoding "
                         "(C1-shaped int8 draft with V151936 -> C2 target, k=4, 512 tokens from a 512-id prompt); "
                         "c5: 64 ragged sequences over a paged int8 KV cache, sharded over the ranks")
    ap.add_argument("--e2e-steps", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--chunk-trace", default=None,
                    help="with --phases: save CTA 0's per-chunk ring events of the last step (.npy)")
    ap.add_argument("--mk", action="store_true",
                    help="run the step as the persistent one-launch kernel (experimental) instead of the kernel sequence")
    ap.add_argument("--phases", action="store_true",
                    help="print the persistent step's per-phase timing (hc_profile_get) after a few steps and exit")
    ap.add_argument("--profile", type=int, default=0,
                    help="run this many decode steps between cudaProfilerStart/Stop after the warm-up and exit "
                         "(for ncu --profile-from-start off)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "linear":
        run_linear(args, local)
        return

    import numpy as np
    import torch

    import hwnpu_b200 as hb
    from hwnpu_b200 import synth

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    if args.workload == "c4":
        run_c4(args, rank, world, local, dist)
        if dist:
            dist.destroy_process_group()
        return
    if args.workload == "c5":
        run_c5(args, rank, world, local, dist)
        return
    W = max(3, args.warmup)
    K = args.steps
    model = build_model(args.workload)
    dev = hb.Device(local)
    lm = dev.load_model(model)
    sess = lm.session(max_context=PROMPT + PASS + W + 8, max_step=8, profile=args.phases,
                      megakernel=args.mk or args.phases)
    prompt = synth.tokens(1, model.cfg.vocab, PROMPT)
    first = sess.greedy(prompt)
    base = sess.pos()
    sess.generate(first, W)
    sess.truncate(base)
    stream = torch.cuda.ExternalStream(sess.stream())
    if args.phases:
        import numpy as np
        acc = None
        for _ in range(8):
            sess.generate(first, 1)
            ph = sess.profile()
            acc = ph if acc is None else acc + ph
        acc /= 8
        cyc = sess.last_cycles
        if args.chunk_trace:
            np.save(args.chunk_trace, sess.last_chunks)
            np.save(args.chunk_trace.replace(".npy", "_unit.npy"), sess.last_unit)
        L = model.cfg.layers
        names = ["qkv", "attention", "o", "gate/up", "down"]
        per = {n: [round(float(x), 3) for x in acc[i:5 * L:5].mean(axis=0)] for i, n in enumerate(names)}
        print(json.dumps({"phase_us_per_layer_inputs_weights_epilogue_barrier": per,
                          "head": acc[5 * L].tolist(), "total_us": float(acc.sum()),
                          "cycles_producer_waited_busy_consumer_waited_busy": [float(x) for x in cyc]}), flush=True)
        return
    if args.profile:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        sess.generate(first, args.profile)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"profiled_steps": args.profile, "launches_per_step": sess.stats()["launches"]}), flush=True)
        return
    launches0 = sess.stats()["launches"]

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local)
    barrier()
    clocks.start()
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
    clk = clocks.stop()
    barrier()

    # e2e: the public per-token call, token in from pinned host memory, choice out, every step
    E = min(args.e2e_steps, PASS)
    tok = first
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(E):
        tok = sess.greedy([tok])
    f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    sess.truncate(base)
    barrier()

    # the dominant kernel: the GEMV over the head (151936 x 2048 int4 g32, the largest launch),
    # timed alone with CUDA events on torch's stream (act quantisation + GEMV of one token)
    import ctypes as C

    from hwnpu_b200 import _abi as A

    h = C.c_void_p()
    A.check(A.lib().hc_linear_load(dev.h, C.byref(model.head.desc()), C.byref(h)))
    x = torch.randn(1, model.cfg.hidden, device="cuda")
    y = torch.empty(1, model.cfg.vocab, device="cuda")
    cs = torch.cuda.current_stream()
    for _ in range(5):
        A.check(A.lib().hc_linear_run(h, C.c_void_p(x.data_ptr()), 1, C.c_void_p(y.data_ptr()), C.c_void_p(cs.cuda_stream)))
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 50
    g0.record(cs)
    for _ in range(reps):
        A.check(A.lib().hc_linear_run(h, C.c_void_p(x.data_ptr()), 1, C.c_void_p(y.data_ptr()), C.c_void_p(cs.cuda_stream)))
    g1.record(cs)
    torch.cuda.synchronize()
    gemv_ms = g0.elapsed_time(g1) / reps
    A.lib().hc_linear_free(h)
    head_bytes = model.head.data.nbytes + model.head.scales.nbytes + (model.head.zeros.nbytes if model.head.zeros is not None else 0)

    from hwnpu_b200 import replicas

    # the job's time is the slowest replica's (every rank runs the same K steps of its own replica)
    t_max = replicas.job_time(ms, dist, "cuda")
    ms_e2e = replicas.job_time(ms_e2e, dist, "cuda")
    cfg = model.cfg
    kv_per_pos = cfg.layers * cfg.kv_heads * cfg.head_dim * 2 * 2
    mean_ctx = PROMPT + (PASS + 1) / 2.0
    bytes_tok = lm.weight_bytes + kv_per_pos * mean_ctx
    peak, peak_kind = peaks()
    value = world * K / (t_max / 1e3)
    per_gpu = K / (ms / 1e3)
    traffic = None
    tf = os.path.join(ROOT, "profiles", "gemv_head_traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get("bytes_per_launch")
        except Exception:
            traffic = None
    ach = head_bytes / (gemv_ms / 1e3) / 1e9
    line = {
        "metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": t_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 x int8(hi+lo) MMA -> int32, f32 scaling", "data": "synthetic (seeded N(0,0.02) weights, uniform ids)",
        "config": workload_config(args),
        "e2e": {"value": world * E / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 16,
                "d2h_bytes_per_step": 4, "api": "hc_step per token (pinned token in, greedy choice out)"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": "gemv_kernel<int4> on the 151936x2048 head (+ its act quantiser)",
                     "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "bytes_per_launch": head_bytes, "ms_per_launch": gemv_ms},
        "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs": bytes_tok * per_gpu / 1e9,
                          "frac": bytes_tok * per_gpu / 1e9 / peak, "ideal_tokens_per_s": peak * 1e9 / bytes_tok},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            tps, dt = cpu_generate(model, 64, 8, os.cpu_count())
            line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                                    "sample": f"8 greedy decode tokens after a 64-id prompt on the oracle ({dt:.1f} s)"}
        except Exception as e:  # the baseline is reported, not required for the GPU number
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    sess.close()
    lm.close()
    dev.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
