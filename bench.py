#!/usr/bin/env python
"""Benchmark: batch-1 INT4 Llama-2-7B decode (the full-model greedy workload).

One step = one decode token through all 32 layers and the LM head
(int4_decoder_controller.cpp:138-234) on seeded synthetic weights in the
reference bank format: a 16-token prompt of ids uniform in [3, 31999], then
greedy tokens, KV capacity 2048, seed 2.  Warm-up steps are the first W
positions; the K timed steps are positions W..W+K-1 (defaults: the 16 prompt
positions, then 128 decode steps).

value  tokens/s over K steps with inputs resident in HBM (embedding rows
       already on the device), CUDA events on the library's stream, max over
       ranks.
e2e    the same K steps through the public C ABI with host data:
       i4d_decode_greedy (token id in, next token id out, 8 B / 12 B copied
       per step); e2e_logits through i4d_decode_token (embedding row in,
       logits, residual and status out every step).
Weights (3.46 GB per token) exceed the 126 MB L2, so no flush is needed.
Further keys: the decode roofline of k_token, a per-stage breakdown from an
instrumented copy, long-context steps (positions 143/1023/2047), config 1
(one Q-shape GEMV), config 2 (one layer at position 511), config 4 (the
attention sweep L = 512..4096), batched prefill and perplexity evaluation,
the reference emulator on the host cores, and the SM clocks sampled during
the timed region.

`--impl reference` times the reference's own CPU implementation (the
emulator compiled from its source into oracle/_ref) on the host cores.
"""
import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 INT4 Llama-2-7B decode tokens/s"
UNIT = "tokens/s"
PROMPT = 16
PREFILL_TOKENS = 128  # prompt length of the prefill measurement
SHARD_GROUP_MAX = 4  # ranks of one bank-sharded group (one bank or more per rank)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="i4d", choices=["i4d", "reference"])
    ap.add_argument("--seed", type=int, default=2)
    ap.add_argument("--kv-capacity", type=int, default=2048)
    ap.add_argument("--cpu-steps", type=int, default=24, help="timed steps of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--soak", type=int, default=400, help="untimed steps before timing (clock steady state)")
    ap.add_argument("--replicas", action="store_true",
                    help="N GPUs decode N independent streams (default for N > 1: one bank-sharded stream)")
    return ap.parse_args()


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="i4d_clocks_", suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
        os.unlink(self.path)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peak():
    try:
        p = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic():
    """DRAM bytes per k_token launch (32 layers) from the committed ncu summary, if any."""
    try:
        return json.load(open(os.path.join(ROOT, "profiles", "k_token_traffic.json")))
    except (OSError, ValueError):
        return None


def write_model_dir(d, banks, emb, lut):
    for p, b in enumerate(banks):
        b.tofile(os.path.join(d, f"model_bank{p}.bin"))
    emb.tofile(os.path.join(d, "embeddings.bin"))
    with open(os.path.join(d, "rope_lut.bin"), "wb") as f:
        f.write(lut)


def cpu_decode(banks, emb, lut, prompt, warmup, steps):
    """The reference's own CPU implementation of the step: the emulator
    compiled from its source (oracle/_ref), all 32 layers and the LM head,
    OpenMP over the host cores.  It runs forward() at positions 0..warmup-1
    untimed, then `steps` timed forwards at positions warmup..warmup+steps-1
    (the GPU arm's positions), feeding the prompt and then its own greedy ids
    (emulator:1608-1682 without the EOS stop).  Returns the measured rate."""
    from oracle import RefEmulator, ref_available
    if not ref_available():
        return None
    tmp = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(prefix="i4d_ref_", dir=tmp) as d:
        write_model_dir(d, banks, emb, lut)
        ref = RefEmulator()
        ref.load(d, 32, 2048)
    tok = prompt[0]
    dt = 0.0
    for pos in range(warmup + steps):
        t0 = time.perf_counter()
        logits, _ = ref.forward(tok, pos)
        if pos >= warmup:
            dt += time.perf_counter() - t0
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else ref.argmax(logits)
    return {"value": steps / dt, "unit": UNIT, "cores": ref.threads(), "kind": "reference",
            "ms_per_step": dt / steps * 1e3, "steps_run": steps, "positions": [warmup, warmup + steps - 1],
            "sample": f"{steps} timed decode steps of the full 32-layer model + LM head at positions "
                      f"{warmup}..{warmup + steps - 1} after {warmup} untimed ones, the same synthetic model "
                      f"and greedy sequence as the GPU arm"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    syn = importlib.import_module("4pe_u250_b200.synth")
    F = importlib.import_module("4pe_u250_b200.formats")
    banks = syn.model_banks(32, args.seed)
    emb = syn.embeddings(args.seed)
    lut = F.generate_rope_lut()
    prompt = np.random.default_rng(args.seed).integers(3, 32000, size=PROMPT).tolist()
    r = cpu_decode(banks, emb, lut, prompt, args.warmup, args.steps)
    if r is None:
        print(json.dumps({"impl": "reference", "unavailable": "the reference emulator (oracle/_ref) was not built"}))
        return
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4xint14/fp32",
            "data": "synthetic", "config": workload_config(args, world),
            "cpu_baseline": r, "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                       "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def long_context_line(ctx, F, args, stream, ev0, ev1, row, d_logits, peak):
    """Decode steps deep into the context (the sharded workload decodes to
    2048): the cache is filled by one prompt prefill of seeded ids, then R
    steps are timed at each position (each rewrites that position's record
    and attends over every earlier one)."""
    out = {"unit": "tokens/s", "positions": {}}
    last = args.kv_capacity - 1
    ids = np.random.default_rng(args.seed + 100).integers(3, 32000, size=last).astype(np.int32)
    ctx.prefill_tokens(0, ids)
    reps = 10
    for p in sorted({143, 1023, last}):
        if p > last:
            continue
        ctx.decode_token_async(p, row(int(ids[p % last])), d_logits.data_ptr())
        ctx.sync()
        ev0.record(stream)
        for _ in range(reps):
            ctx.decode_token_async(p, row(int(ids[p % last])), d_logits.data_ptr())
        ev1.record(stream)
        ctx.sync()
        ms = ev0.elapsed_time(ev1) / reps
        nbytes = F.token_bytes(p)
        out["positions"][str(p)] = {"tok_s": 1000.0 / ms, "ms_per_step": ms, "bytes_per_token": nbytes,
                                    "frac_of_peak": nbytes / (ms * 1e-3) / 1e9 / peak}
    return out


def layer_line(pkg, F, syn, lut, emb, device, peak):
    """Config 2: one decoder layer at position 511 over 511 prior KV records
    (the layer of forward(), emulator:727-783).  The step of a 2-layer model
    minus that of a 1-layer model at the same position is one layer's time
    (the final norm and LM head cancel); the caches are filled by a prefill of
    511 seeded ids.  Algorithmic bytes: the layer's weights and gammas plus
    512 records per head."""
    import torch
    ids = np.random.default_rng(1).integers(3, 32000, size=512).astype(np.int32)
    d_emb = torch.from_numpy(emb).to(f"cuda:{device}")
    out = {}
    for layers in (1, 2):
        with pkg.Context(device=device, num_layers=layers, kv_capacity=512) as c:
            c.load_banks(syn.model_banks(layers, 1))
            c.load_rope(lut)
            c.load_embeddings(emb)
            c.prefill_tokens(0, ids[:511])
            d_logits = torch.empty(F.PADDED_VOCAB, dtype=torch.float32, device=f"cuda:{device}")
            row = d_emb.data_ptr() + int(ids[511]) * 4096 * 4
            s = torch.cuda.ExternalStream(c.stream_handle())
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            for _ in range(10):
                c.decode_token_async(511, row, d_logits.data_ptr())
            c.sync()
            reps = 50
            e0.record(s)
            for _ in range(reps):
                c.decode_token_async(511, row, d_logits.data_ptr())
            e1.record(s)
            c.sync()
            out[layers] = e0.elapsed_time(e1) / reps
    us = (out[2] - out[1]) * 1e3
    nbytes = 105971712 + 2 * 4096 * 4 + 512 * 32 * 261
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": "config2: one decoder layer at position 511 over 511 prior KV records (2-layer step minus 1-layer step)",
            "us_per_layer": us, "bytes": nbytes, "gbs": gbs, "frac_of_peak": gbs / peak,
            "step_ms": {"1_layer": out[1], "2_layers": out[2]}}


def gemv_line(ctx, F, peak, peak_kind, streams, max_over_ranks):
    """The single INT4 GEMV of the Q-projection shape (4096 x 4096 in four
    input-column bank shards, 8,650,752 B of nibbles and Q1.15 scales): the
    op of sharded_gemv_4pe (emulator:216-264) through the library's GEMV
    kernel, one launch per GEMV, each on the next layer's Q matrix (32
    matrices, 277 MB > the 126 MB L2, so every launch streams from HBM)."""
    reps = 320
    ctx.profile_gemv(F.MODE_Q, 32)  # warm-up
    ms = max_over_ranks(ctx.profile_gemv(F.MODE_Q, reps))
    nbytes = 4096 * 4096 // 2 + 4096 * 32 * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "config1: one Q-shape INT4 GEMV y = Wx, W 4096 x 4096 in the packer's 4-bank tile layout",
            "value": streams * gbs, "unit": "GB/s", "us_per_gemv": ms * 1e3, "bytes_per_gemv": nbytes,
            "launches": reps, "frac_of_peak": gbs / peak, "peak": peak, "peak_kind": peak_kind,
            "l2": "32 distinct matrices in rotation (277 MB > 126 MB L2)"}


def attention_line(pkg, F, syn, lut, device, peak, peak_kind):
    """The attention-only sweep: RoPE + INT8-KV fixed-point online softmax for
    32 heads x 128 (swiftkv_attention_4pe, emulator:602-714) at context
    lengths 512..4096 (position L-1).  The cache is filled by the attention
    step itself over 16 seeded N(0,1) q/k/v rows taken to Q15.17; each timed
    step reads 32 * L records (261 algorithmic bytes each)."""
    import torch
    from oracle import Oracle
    orc = Oracle()
    rng = np.random.default_rng(3)
    rows = np.stack([orc.float_to_q17(rng.standard_normal(3 * 4096).astype(np.float32)) for _ in range(16)])
    qkv = torch.from_numpy(rows.astype(np.int32)).to(f"cuda:{device}")
    out = {"workload": "config4: attention of one layer, 32 heads x 128, INT8 KV, L = 512/1024/2048/4096",
           "unit": "GB/s", "peak": peak, "peak_kind": peak_kind, "L": {}}
    with pkg.Context(device=device, num_layers=1, kv_capacity=4096) as actx:
        actx.load_rope(lut)
        actx.profile_attention(0, 4095, qkv.data_ptr(), 16, 1)  # writes the records of positions 0..4094
        for L in (512, 1024, 2048, 4096):
            ms = actx.profile_attention(0, L - 1, qkv.data_ptr(), 0, 50)
            nbytes = 32 * L * 261
            gbs = nbytes / (ms * 1e-3) / 1e9
            out["L"][str(L)] = {"us": ms * 1e3, "bytes": nbytes, "gbs": gbs, "frac_of_peak": gbs / peak}
    out["value"] = out["L"]["4096"]["gbs"]
    return out


def shard_group_size(world):
    """Ranks per bank-sharded group: all of them up to 4 (the banks), else
    groups of 4, each decoding its own stream."""
    return world if world <= SHARD_GROUP_MAX else SHARD_GROUP_MAX


def workload_config(args, world):
    g = shard_group_size(world)
    par = ("1gpu" if world == 1 else f"replicas{world}" if args.replicas else
           f"bank-shard{g}" if g == world else f"bank-shard{g}x{world // g}")
    return {"workload": "config3: full 32-layer INT4 Llama-2-7B decode, 16-token prompt then greedy, "
                        "KV capacity 2048, seed 2",
            "layers": 32, "kv_capacity": args.kv_capacity, "positions": [args.warmup, args.warmup + args.steps - 1],
            "parallelism": par,
            "l2": "weights 3.46 GB/token exceed the 126 MB L2 (no flush needed)"}


def main():
    args = parse()
    world, rank, local = dist_setup()
    if args.impl == "reference":
        if world > 1:
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))
        run_reference(args, world, rank)
        return
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    pkg = importlib.import_module("4pe_u250_b200")
    syn = importlib.import_module("4pe_u250_b200.synth")
    F = pkg.formats
    total = args.warmup + args.steps
    assert total <= args.kv_capacity

    shard = world > 1 and not args.replicas
    gsize = shard_group_size(world) if shard else 1
    if shard and (world % gsize or gsize not in (2, 4)):
        raise SystemExit(f"bank sharding needs 2, 4 or a multiple of 4 GPUs; use --replicas for {world}")
    group = None
    if shard and gsize < world:  # every rank creates every group, in the same order
        groups = [dist.new_group(list(range(g0, g0 + gsize))) for g0 in range(0, world, gsize)]
        group = groups[rank // gsize]
    banks = syn.model_banks(32, args.seed)
    emb = syn.embeddings(args.seed)
    lut = F.generate_rope_lut()
    if shard:
        ctx = pkg.Context(device=local, num_layers=32, kv_capacity=args.kv_capacity, rank=rank % gsize, world=gsize)
    else:
        ctx = pkg.Context(device=local, num_layers=32, kv_capacity=args.kv_capacity)
    ctx.load_banks(banks)
    ctx.load_rope(lut)
    ctx.load_embeddings(emb)
    if shard:
        ctx.attach_peers(group)
    stream = torch.cuda.ExternalStream(ctx.stream_handle())
    prompt = np.random.default_rng(args.seed).integers(3, 32000, size=PROMPT).tolist()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- e2e through the public C ABI: the greedy step (token id in, next id
    # out: i4d_decode_greedy), then the logits contract (i4d_decode_token:
    # embedding row in, 32256 logits out, host argmax) on the same sequence ----
    tokens, nxt = [], None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for pos in range(total):
        if pos == args.warmup:
            barrier()
            ev0.record(stream)
        tok = prompt[pos] if pos < PROMPT else nxt
        tokens.append(tok)
        nxt, _ = ctx.decode_greedy(pos, tok)
    ev1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1))
    last_logits = None
    for pos in range(total):
        if pos == args.warmup:
            barrier()
            ev0.record(stream)
        tok = tokens[pos]
        last_logits = ctx.decode_token(pos, emb[tok * 4096:(tok + 1) * 4096])
        if pos + 1 < total and pos + 1 >= PROMPT:
            assert int(np.argmax(last_logits[:F.VOCAB])) == tokens[pos + 1]  # same greedy sequence
    ev1.record(stream)
    barrier()
    e2e_logits_ms = max_over_ranks(ev0.elapsed_time(ev1))

    # ---- device-resident replay of the same token sequence ----
    d_emb = torch.from_numpy(emb).to("cuda")
    d_logits = torch.empty(F.PADDED_VOCAB, dtype=torch.float32, device="cuda")
    row = lambda t: d_emb.data_ptr() + t * 4096 * 4  # noqa: E731
    for pos in range(args.warmup):
        ctx.decode_token_async(pos, row(tokens[pos]), d_logits.data_ptr())
    ctx.sync()
    clocks = Clocks(local)
    clocks.start()
    for i in range(args.soak):  # untimed, same positions: brings clocks to steady state
        pos = args.warmup + i % args.steps
        ctx.decode_token_async(pos, row(tokens[pos]), d_logits.data_ptr())
    ctx.sync()
    barrier()
    ev0.record(stream)
    for pos in range(args.warmup, total):
        ctx.decode_token_async(pos, row(tokens[pos]), d_logits.data_ptr())
    ev1.record(stream)
    ctx.sync()
    barrier()
    clk = clocks.stop()
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1))
    replay_ok = bool(np.array_equal(d_logits.cpu().numpy(), last_logits))

    # ---- device time of the token kernel alone (events around the launch) ----
    mid = args.warmup + args.steps // 2
    if shard:  # the per-kernel hooks run one context alone; use the replay time
        tok_ms = dev_ms / args.steps
        breakdown = {}
    else:
        tok_ms = []
        for _ in range(5):
            p = ctx.profile_token(mid, row(tokens[mid]))
            tok_ms.append(p["token"][0])
        tok_ms = statistics.median(tok_ms)
        breakdown = ctx.token_breakdown(mid, row(tokens[mid]))
    peak, peak_kind = measured_peak()
    # A shard streams its banks' share of the bytes: per-GPU bandwidth.
    achieved = F.token_bytes(mid) / gsize / (tok_ms * 1e-3) / 1e9
    traffic = committed_traffic()

    streams = world // gsize  # a sharded group decodes one stream
    value = streams * args.steps / (dev_ms * 1e-3)
    e2e = streams * args.steps / (e2e_ms * 1e-3)
    e2e_logits = streams * args.steps / (e2e_logits_ms * 1e-3)
    launches_per_step = 2  # k_set_pos + k_token
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if shard and gsize == world else "weak", "vs_baseline": None, "dtype": "int4xint14/fp32",
        "data": "synthetic", "config": workload_config(args, world),
        "e2e": {"value": e2e, "unit": UNIT, "api": "i4d_decode_greedy (token id in, next token id out)",
                "h2d_bytes_per_step": 4 + 4, "d2h_bytes_per_step": 8 + 4, "ms_per_step": e2e_ms / args.steps},
        "e2e_logits": {"value": e2e_logits, "unit": UNIT,
                       "api": "i4d_decode_token (embedding row in, 32256 logits out, host argmax)",
                       "h2d_bytes_per_step": 4096 * 4 + 4, "d2h_bytes_per_step": F.PADDED_VOCAB * 4 + 4096 * 4 + 4,
                       "ms_per_step": e2e_logits_ms / args.steps},
        "roofline": {"bound": "hbm", "kernel": "k_token (persistent decode step, 1 launch per token" +
                               (f" on each of {gsize} bank shards; achieved = per-GPU share of the bytes)" if shard
                                else ")"),
                     "achieved": achieved, "peak": peak,
                     "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback", "unit": "GB/s", "frac": achieved / peak,
                     "traffic": (traffic["bytes_per_launch"] if traffic and not shard else None),
                     "algorithmic_bytes_per_launch": F.token_bytes(mid) // gsize,
                     "kernel_ms": tok_ms},
        "token_roofline": {"bytes_per_token": F.token_bytes(mid), "achieved_gbs":
                           F.token_bytes(mid) / (dev_ms / args.steps * 1e-3) / 1e9,
                           "frac": F.token_bytes(mid) / (dev_ms / args.steps * 1e-3) / 1e9 / peak},
        "token_kernel_breakdown_us": {k: round(v, 2) for k, v in breakdown.items()},
        "gpu_launches": launches_per_step * args.steps,
        "replay_matches_e2e": replay_ok,
        "clocks": clk,
    }
    # ---- batched prompt prefill (i4d_prefill_tokens) of the same token
    # sequence: it rewrites the same KV records bit for bit, and its greedy
    # next id must be the decoded continuation ----
    if not shard:
        n_pf = min(PREFILL_TOKENS, total - 1)
        ids = np.asarray(tokens[:n_pf], np.int32)
        ctx.prefill_tokens(0, ids)  # warm-up
        barrier()
        reps = 3
        ev0.record(stream)
        for _ in range(reps):
            nxt_pf, _ = ctx.prefill_tokens(0, ids)
        ev1.record(stream)
        barrier()
        pf_ms = max_over_ranks(ev0.elapsed_time(ev1)) / reps
        batches = -(-n_pf // 32)  # prompt tokens per batch
        line["prefill"] = {"value": streams * n_pf / (pf_ms * 1e-3), "unit": "prompt tokens/s", "tokens": n_pf,
                           "ms": pf_ms, "api": "i4d_prefill_tokens (token ids in, greedy next id out)",
                           "h2d_bytes": 8 * n_pf, "d2h_bytes": 8 + 4 * batches,
                           "matches_decode": bool(nxt_pf == tokens[n_pf]) if n_pf >= PROMPT else None}
        # ---- perplexity terms of the same tokens (i4d_eval_nll: n - 1 positions) ----
        ctx.eval_nll(ids)
        barrier()
        ev0.record(stream)
        for _ in range(reps):
            ctx.eval_nll(ids)
        ev1.record(stream)
        barrier()
        ev_ms = max_over_ranks(ev0.elapsed_time(ev1)) / reps
        line["perplexity_eval"] = {"value": streams * (n_pf - 1) / (ev_ms * 1e-3), "unit": "positions/s",
                                   "positions": n_pf - 1, "ms": ev_ms,
                                   "api": "i4d_eval_nll (token ids in, one NLL per position out)"}
    if not shard:
        line["long_context"] = long_context_line(ctx, F, args, stream, ev0, ev1, row, d_logits, peak)
        line["gemv"] = gemv_line(ctx, F, peak, peak_kind, streams, max_over_ranks)
        line["layer"] = layer_line(pkg, F, syn, lut, emb, local, peak)
        line["attention"] = attention_line(pkg, F, syn, lut, local, peak, peak_kind)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_decode(banks, emb, lut, prompt, args.warmup, min(args.steps, args.cpu_steps))
        if r is not None:
            line["cpu_baseline"] = r
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
