"""bench.py — MoE tokens/s of the Drama3-like routed-expert FFN stack on 1, 2, 4 or 8 B200s.

Contract (the driver's): `python bench.py --gpus N --steps K --warmup W [--impl reference]` prints ONE JSON line.
A step is one pass of config 5's stack over one batch: 48 layers of b200_moe_ffn (gate|up MUL_MAT_ID 2048 -> 1536,
SwiGLU, down MUL_MAT_ID 768 -> 2048, router-weighted sum; TextModel::experts, src/families/drama3/text-model.cpp:198-221)
over 128 Q8_0 experts, top-8 routes of N(0, 1) router logits, 256 N(0, 1) tokens, each layer's output the next layer's
input. With N GPUs the experts are split across the ranks (expert parallelism: rank r holds experts [r E/N, (r+1) E/N)
of every layer) and the ranks' partial sums are added over NVLink every layer, so every rank holds the full layer
output; the same 256 tokens at every N (strong scaling). `value` = tokens/s of the whole job (256 x K / the
max-over-ranks device time).

At N = 1 the line also carries the other configurations of BASELINE.json as side keys (`configs`): config 2's decode
step, config 1's single GEMV, config 3's decode step and prefill (as a fraction of the measured int8 tensor peak),
config 4's batched stack and single large GEMVs; and, in the CPU-baseline leg, a parity check of the timed stack's
first layer against the CPU oracle on the same weights and inputs.

`--impl reference` times the CPU restatement of ggml's CPU backend (oracle/; ggml itself is absent from the reference
checkout) on the same stack — all 48 layers, chained — for a sample of the tokens, with every host thread.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

UNIT = "tok/s"
MOE = {"n_expert": 128, "top_k": 8, "hidden": 2048, "ffn": 768, "n_layer": 48, "tokens": 256}
MOE_METRIC = "MoE tok/s, Drama3-like MoE FFN stack (48 layers x 128 Q8_0 experts, top-8, 2048<->768), 256 tokens per step"
MOE_WORKLOAD = ("config 5: 48 chained layers of b200_moe_ffn (gate|up 2048->1536, SwiGLU, down 768->2048, weighted sum) over "
                "128 Q8_0 experts, top-8 of N(0,1) router logits, 256 N(0,1) tokens")
# kernels of this library launched per MoE layer (route+quantize, gate|up with SwiGLU, down, combine; at N > 1 the
# combine also adds the ranks' partial sums over NVLink, or an NCCL all-reduce follows it)
MOE_KERNELS_PER_LAYER = 6

Q8_0, Q4_K, Q6_K = 8, 12, 14
# Decoder stacks of BASELINE.json: the Qwen3-TTS 0.6B talker (config 2), the Qwen3-ASR 1.7B-shaped decoder (config 3)
DECODERS = {
    "tts06": dict(n_layer=28, hidden=1024, n_head=16, n_kv_head=8, head_dim=128, ffn=3072, n_vocab=3072,
                  type_attn=Q8_0, type_ffn_up=Q8_0, type_ffn_down=Q8_0, type_head=Q8_0),
    "asr17": dict(n_layer=28, hidden=2048, n_head=16, n_kv_head=8, head_dim=128, ffn=6144, n_vocab=151936,
                  type_attn=Q4_K, type_ffn_up=Q4_K, type_ffn_down=Q6_K, type_head=Q6_K),
}


def decoder_tensor_shapes(c):
    """(type, K, N) of each matrix of one decoder layer, and of the head."""
    attn, kv = c["n_head"] * c["head_dim"], c["n_kv_head"] * c["head_dim"]
    h, f = c["hidden"], c["ffn"]
    return {"attn_q": (c["type_attn"], h, attn), "attn_k": (c["type_attn"], h, kv), "attn_v": (c["type_attn"], h, kv),
            "attn_o": (c["type_attn"], attn, h), "ffn_gate": (c["type_ffn_up"], h, f), "ffn_up": (c["type_ffn_up"], h, f),
            "ffn_down": (c["type_ffn_down"], f, h), "output": (c["type_head"], h, c["n_vocab"])}


def load_package():
    import importlib.util

    name = "speechcpp_b200"
    if name in sys.modules:
        return sys.modules[name]
    path = os.path.join(ROOT, "speech.cpp_b200", "__init__.py")
    spec = importlib.util.spec_from_file_location(name, path, submodule_search_locations=[os.path.dirname(path)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def peak_fields(peak, kind):
    return {"peak": peak, "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else "fallback 6650 GB/s"}


def host_threads():
    """Every host thread this process may run on (torchrun sets OMP_NUM_THREADS=1 for its ranks; the CPU legs pass
    this count to the oracle explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# DRAM bytes (read + write) of one decoder_mk_kernel launch of the config-2 step, from an ncu capture of that launch
# (dram__bytes_read.sum + dram__bytes_write.sum).
DECODE_TRAFFIC = 471652608 + 4275968
# DRAM bytes of one MoE layer's two gemm_q8_0_tc_grouped_kernel launches (gate|up + down) from an ncu capture of the
# 2-layer case on one GPU; the step's traffic scales with its layers and, across N ranks, divides by N.
MOE_TRAFFIC_PER_LAYER = 434762496 + 12986368 + 216577024 + 12018688


class Clocks:
    """Samples nvidia-smi during the timed region (SM clock, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.p:
            time.sleep(0.25)
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except Exception:
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def moe_routes(c, seed=11):
    """Per layer: router logits N(0, 1) -> softmax -> top-k (ties broken by a seeded permutation of the experts)
    -> weights renormalised over the chosen k. Returns ids int32 [L, T, k], w float32 [L, T, k]."""
    import numpy as np

    rng = np.random.default_rng(seed)
    L, T, E, k = c["n_layer"], c["tokens"], c["n_expert"], c["top_k"]
    ids = np.empty((L, T, k), dtype=np.int32)
    w = np.empty((L, T, k), dtype=np.float32)
    for l in range(L):
        logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
        p = np.exp(logits - logits.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        rank = rng.permutation(E)
        order = np.lexsort((np.broadcast_to(rank, (T, E)), -p), axis=1)[:, :k]
        ids[l] = order
        sel = np.take_along_axis(p, order, 1)
        w[l] = sel / sel.sum(1, keepdims=True)
    return ids, w


class CpuMoe:
    """The CPU oracle's MoE stack (oracle/: ggml-CPU semantics restated; the reference's own CPU path): per layer the
    gate|up MUL_MAT_ID, SwiGLU and the down MUL_MAT_ID, then the router-weighted sum in slot order, with `nthreads`
    host threads. Used only by the reference arm, the CPU-baseline leg and its parity check.

    For timing, one layer's worth of random valid Q8_0 expert blocks (641 MB, larger than any CPU cache) stands in for
    every layer's experts: the CPU's time per layer does not depend on the weight values, and every layer still
    streams its experts from DRAM. The routes are config 5's own (all 48 layers); `tokens` of the 256 run (a bounded
    sample: the oracle's cost is the same for every (token, slot) pair)."""

    def __init__(self, c, tokens, nthreads):
        import numpy as np

        from oracle import oracle

        self.o, self.c, self.nthreads, self.tokens = oracle, c, nthreads, tokens
        rng = np.random.default_rng(17)
        H, F, E = c["hidden"], c["ffn"], c["n_expert"]

        def blocks(rows, K):
            b = rng.integers(-127, 128, size=(rows * (K // 32), 34), dtype=np.int8).view(np.uint8)
            b[:, :2] = (rng.random(rows * (K // 32)) * 2e-4 + 1e-4).astype(np.float16).view(np.uint8).reshape(-1, 2)
            return b.reshape(rows, -1)

        self.gu, self.dn = blocks(E * 2 * F, H), blocks(E * H, F)
        ids, w = moe_routes(c)
        self.ids, self.w = ids[:, :tokens], w[:, :tokens]
        self.x = rng.normal(0, 1, size=(tokens, H)).astype(np.float32)

    def layer(self, gu, dn, x, ids, w):
        import numpy as np

        o, c = self.o, self.c
        H, F, E = c["hidden"], c["ffn"], c["n_expert"]
        gu_out = o.mul_mat_id(o.Q8_0, gu, H, 2 * F, E, x[:, None, :], ids, self.nthreads)
        g, u = gu_out[..., :F], gu_out[..., F:]
        act = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
        dn_out = o.mul_mat_id(o.Q8_0, dn, F, H, E, act, ids, self.nthreads)
        out = np.zeros((x.shape[0], H), dtype=np.float32)
        for s in range(ids.shape[1]):
            out = (out + dn_out[:, s] * w[:, s:s + 1]).astype(np.float32)
        return out

    def step(self):
        x = self.x
        for l in range(self.c["n_layer"]):
            x = self.layer(self.gu, self.dn, x, self.ids[l], self.w[l])
        return x

    def sample_text(self, steps):
        return (f"{steps} steps of all {self.c['n_layer']} chained layers for {self.tokens} of the {self.c['tokens']} tokens "
                f"(their config-5 routes), one layer's random Q8_0 experts (641 MB) standing in for every layer's")


def cpu_moe_rate(c, tokens, nthreads, warmup, steps):
    """Tokens/s of the oracle's 48-layer stack over `tokens` tokens: total tokens / total time of `steps` steps."""
    cm = CpuMoe(c, tokens, nthreads)
    for _ in range(warmup):
        cm.step()
    times = []
    for _ in range(steps):
        a = time.perf_counter()
        cm.step()
        times.append(time.perf_counter() - a)
    return tokens * steps / sum(times), cm.sample_text(steps), times


def moe_parity(pkg, ctx, gu, dn, x, ids, w, got, nthreads):
    """Layer 0 of the timed GPU stack against the CPU oracle on the same weights (read back from the device as GGUF
    bytes) and inputs: per-token cosine similarity (bar >= 0.9999, the decoder-stack bar: the SwiGLU output is
    re-quantized) and max |err| / max |ref|."""
    import numpy as np

    from oracle import oracle

    c = MOE
    H, F, E = c["hidden"], c["ffn"], c["n_expert"]
    gub = ctx.get_weight(gu).reshape(E * 2 * F, -1)
    dnb = ctx.get_weight(dn).reshape(E * H, -1)
    cm = CpuMoe.__new__(CpuMoe)
    cm.o, cm.c, cm.nthreads = oracle, c, nthreads
    want = cm.layer(gub, dnb, x, ids, w)
    cos = (got * want).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
    return {"check": "layer 0 of the timed stack vs the CPU oracle on the same weights and inputs", "tokens": int(x.shape[0]),
            "min_token_cosine": float(cos.min()), "bar": 0.9999, "max_abs_err_over_max_abs": float(np.abs(got - want).max() / np.abs(want).max()),
            "pass": bool(cos.min() >= 0.9999)}


def run_reference(args):
    """The reference arm: the CPU oracle's stack, rank 0 only (the other ranks exit at once), all host threads."""
    world, rank, local = dist_setup()
    if rank != 0:
        return 0
    nthreads = host_threads()
    t0 = time.perf_counter()
    value, sample, times = cpu_moe_rate(MOE, args.ref_tokens, nthreads, args.warmup, args.steps)
    wall = time.perf_counter() - t0
    emit({
        "impl": "reference", "metric": MOE_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * MOE["tokens"] / value, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8xint8->int32, f32 accumulate", "data": "synthetic",
        "config": {"workload": MOE_WORKLOAD, "global_batch": MOE["tokens"], "parallelism": f"cpu, {nthreads} threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": wall, "step_s_median": statistics.median(times),
        "note": "CPU restatement of ggml's CPU quantized vec_dot (oracle/); ggml itself is absent from the reference checkout. "
                "ms_per_step is for the full 256 tokens at this rate",
    })
    return 0


def moe_weights(pkg, ctx, c, e0, E_local):
    """Layer weights of experts [e0, e0 + E_local): gate|up [H, 2F, E_local] and down [F, H, E_local], Q8_0. Each
    expert's values are N(0, 0.02) from a generator seeded by (layer, expert), quantized on the device by the backend's
    Q8_0 quantizer, so a shard holds exactly the bytes the same experts have on one GPU."""
    import torch

    H, F = c["hidden"], c["ffn"]
    g = torch.Generator(device="cuda")
    gus, dns = [], []
    rs_gu, rs_dn = 2 * F * pkg.row_size(pkg.Q8_0, H), H * pkg.row_size(pkg.Q8_0, F)
    for l in range(c["n_layer"]):
        gu = ctx.weight(pkg.Q8_0, H, 2 * F, E_local)
        dn = ctx.weight(pkg.Q8_0, F, H, E_local)
        for j in range(E_local):
            g.manual_seed(1_000_003 * l + e0 + j)
            ctx.set_weight(gu, ctx.quantize_rows(pkg.Q8_0, torch.randn((2 * F, H), generator=g, device="cuda") * 0.02), offset=j * rs_gu)
            ctx.set_weight(dn, ctx.quantize_rows(pkg.Q8_0, torch.randn((H, F), generator=g, device="cuda") * 0.02), offset=j * rs_dn)
        gus.append(gu)
        dns.append(dn)
    ctx.synchronize()
    return gus, dns


def run_moe(args, pkg, ctx, dist, world, rank, local):
    """Expert parallelism: rank r holds experts [r E/N, (r+1) E/N) of every layer; activations and routes are
    replicated (the router runs on every rank), so dispatch moves nothing; each rank computes its experts' pairs, and
    the ranks' partial sums are added every layer (in the combine kernel over NVLink peer memory, or by an NCCL
    all-reduce), so every rank holds the next layer's input. The 48-layer step is captured in one CUDA graph."""
    import numpy as np
    import torch

    c = dict(MOE, n_layer=args.moe_layers)
    E, T, H, k, L = c["n_expert"], c["tokens"], c["hidden"], c["top_k"], c["n_layer"]
    import importlib

    ep = importlib.import_module(pkg.__name__ + ".expert_parallel")
    e0, E_local = ep.expert_shard(E, world, rank)
    gus, dns = moe_weights(pkg, ctx, c, e0, E_local)
    combine = args.moe_combine if world > 1 else "local"
    peer = ep.PeerCombine(ctx, dist.group.WORLD, T, H) if combine == "peer" else None
    moe = ep.ExpertParallelMoe(ctx, zip(gus, dns), e0, E, group=dist.group.WORLD if dist else None, peer=peer)
    ids_h, w_h = moe_routes(c)
    ids = torch.from_numpy(ids_h).cuda()
    wts = torch.from_numpy(w_h).cuda()
    xs = [torch.randn((T, H), generator=torch.Generator(device="cuda").manual_seed(7), device="cuda")]
    xs += [torch.empty((T, H), device="cuda") for _ in range(L)]
    stream = ctx.torch_stream()

    def step():
        moe.step(xs, ids, wts)

    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
    torch.cuda.synchronize()
    ctx.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    ctx.synchronize()  # any device-side error (a timed-out wait) surfaces here

    steps = args.steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(steps):
                graph.replay()
            ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / steps
    value = T * steps / (ms / 1000.0)

    # end to end: pinned host activations and routes in, the last layer's output out, every step
    x_pin = torch.empty((T, H), pin_memory=True).copy_(xs[0].cpu())
    ids_pin = torch.from_numpy(ids_h).pin_memory()
    w_pin = torch.from_numpy(w_h).pin_memory()
    out_pin = torch.empty((T, H), pin_memory=True)

    def e2e_step():
        with torch.cuda.stream(stream):
            xs[0].copy_(x_pin, non_blocking=True)
            ids.copy_(ids_pin, non_blocking=True)
            wts.copy_(w_pin, non_blocking=True)
            graph.replay()
            out_pin.copy_(xs[L], non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    if dist:
        dist.barrier()
    e0v, e1v = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0v.record(stream)
    for _ in range(steps):
        e2e_step()
    e1v.record(stream)
    e1v.synchronize()
    ems = e0v.elapsed_time(e1v)
    if dist:
        dist.barrier()
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    del graph
    torch.cuda.synchronize()
    ctx.synchronize()
    if peer is not None:
        peer.close()
    # what the parity check needs: layer 0's input and output (the graph's last replay) and its weights
    keep = {"x0": xs[0].cpu().numpy(), "y0": xs[1].cpu().numpy(), "ids0": ids_h[0], "w0": w_h[0], "weights": gus + dns}
    wbytes = sum(w.nbytes for w in gus) + sum(w.nbytes for w in dns)
    peak, peak_kind = peaks()
    achieved = wbytes / (ms_step / 1000.0) / 1e9
    res = {
        "metric": MOE_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8xint8->int32, f32 accumulate", "data": "synthetic",
        "config": {"workload": MOE_WORKLOAD if L == MOE["n_layer"] else MOE_WORKLOAD.replace("48 chained", f"{L} chained"),
                   "global_batch": T, "seq_len": 1,
                   "parallelism": (f"expert-parallel x{world}, " + ("partial sums added by the combine kernel over NVLink peer memory"
                                   if combine == "peer" else "NCCL all-reduce of the partial sums")) if world > 1 else "single",
                   "l2": f"expert weights {wbytes / 1e9:.1f} GB per GPU > 126 MB L2 (each step streams them from HBM; no flush needed)"},
        "roofline": dict({"bound": "hbm", "kernel": "the MoE layer stack per GPU (gemm_q8_0_tc_grouped_kernel, the dominant kernel, "
                                                    "and the route / SwiGLU / combine kernels)",
                          "achieved": achieved, "unit": "GB/s", "frac": achieved / peak,
                          "algorithmic_bytes_per_step": wbytes, "algorithmic_unit": "expert weight bytes of this GPU's shard per step",
                          "traffic": MOE_TRAFFIC_PER_LAYER * L // world,
                          "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the expert GEMMs of a 2-layer "
                                            "one-GPU capture, scaled to the step's layers and this GPU's share"}, **peak_fields(peak, peak_kind)),
        "e2e": {"value": T * steps / (ems / 1000.0), "unit": UNIT, "h2d_bytes_per_step": T * H * 4 + ids_h[0].nbytes * L + w_h[0].nbytes * L,
                "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": MOE_KERNELS_PER_LAYER * L * steps,
        "clocks": clk.summary(),
    }
    return res, keep


def make_decoder(pkg, ctx, seed, name="tts06"):
    """A decoder stack of DECODERS[name] with device-generated random weights: Q8_0 tensors are N(0, 0.02) quantized
    on the device by b200_quantize_rows; K-quant tensors are random valid blocks."""
    import torch

    c = DECODERS[name]
    d = pkg.Decoder(ctx, **c)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    sh = decoder_tensor_shapes(c)

    def blocks(t, k, rows):
        if t == pkg.Q8_0:
            return ctx.quantize_rows(t, torch.randn((rows, k), generator=g, device="cuda", dtype=torch.float32) * 0.02)
        return _random_kquant_blocks(t, rows, k, g)

    names = ["attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down"]
    for l in range(c["n_layer"]):
        for i, n in enumerate(names):
            t, k, rows = sh[n]
            d.set_tensor(l, i, blocks(t, k, rows))
        d.set_tensor(l, pkg.DEC_ATTN_NORM, 1.0 + 0.1 * torch.randn(c["hidden"], generator=g, device="cuda"))
        d.set_tensor(l, pkg.DEC_FFN_NORM, 1.0 + 0.1 * torch.randn(c["hidden"], generator=g, device="cuda"))
    t, k, rows = sh["output"]
    d.set_tensor(0, pkg.DEC_OUTPUT, blocks(t, k, rows))
    d.set_tensor(0, pkg.DEC_OUTPUT_NORM, 1.0 + 0.1 * torch.randn(c["hidden"], generator=g, device="cuda"))
    ctx.synchronize()
    return d, c


def config2_decode(pkg, ctx, stream, steps, warmup, seed=1234):
    """Config 2: decode tokens/s of the Qwen3-TTS 0.6B talker step (28 x {q|k|v 1024->4096, o 2048->1024,
    gate|up 1024->6144, down 3072->1024} + head 1024->3072, Q8_0, batch 1), one persistent launch per step; and the
    same end to end through b200_decoder_step_host (input row in, logits out, every step)."""
    import numpy as np
    import torch

    dec, c = make_decoder(pkg, ctx, seed=seed)
    x = torch.randn(c["hidden"], generator=torch.Generator(device="cuda").manual_seed(7), device="cuda")
    logits = torch.empty(c["n_vocab"], device="cuda")
    for _ in range(max(warmup, 3)):
        dec.step_raw(x.data_ptr(), logits.data_ptr())
    ctx.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        dec.step_raw(x.data_ptr(), logits.data_ptr())
    ev1.record(stream)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    xh = x.cpu().numpy()
    out = np.empty(c["n_vocab"], dtype=np.float32)
    for _ in range(2):
        dec.step_host(xh, out)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        dec.step_host(xh, out)
    e1.record(stream)
    e1.synchronize()
    ems = e0.elapsed_time(e1) / steps
    wb, launches = dec.weight_bytes, dec.launches
    del dec
    peak, kind = peaks()
    gbs = wb / ms / 1e6
    return {"workload": "config 2: qwen3-tts-0.6b talker decode step, 28 x {q|k|v 1024->4096, o 2048->1024, gate|up 1024->6144, "
                        "down 3072->1024} + head 1024->3072, Q8_0, batch 1", "steps": steps, "ms_per_step": ms, "tok_s": 1000.0 / ms,
            "e2e_tok_s": 1000.0 / ems, "e2e_h2d_bytes_per_step": c["hidden"] * 4, "e2e_d2h_bytes_per_step": c["n_vocab"] * 4,
            "weight_bytes": wb, "launches_per_step": launches, "gbs": gbs, "frac": gbs / peak, "bound": "hbm",
            "kernel": "decoder_mk_kernel (the whole step, one launch)", "traffic": DECODE_TRAFFIC,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one decoder_mk_kernel launch", **peak_fields(peak, kind)}


def config1_gemv(pkg, ctx, stream, copies=64, calls=256, reps=10):
    """Config 1's single product (Q8_0, K = 1024, N = 3072, one activation row): 256 back-to-back b200_mul_mat calls
    in one CUDA graph over 64 distinct weight copies (214 MB > L2), so every call streams its weights from HBM."""
    import ctypes

    import torch

    K, N = 1024, 3072
    g = torch.Generator(device="cuda").manual_seed(11)
    ws = [ctx.weight(pkg.Q8_0, K, N, data=ctx.quantize_rows(pkg.Q8_0, torch.randn((N, K), generator=g, device="cuda") * 0.02))
          for _ in range(copies)]
    x = torch.randn((1, K), generator=g, device="cuda")
    ys = [torch.empty((1, N), device="cuda") for _ in range(copies)]
    ctx.synchronize()
    fn, h = ctx.L.b200_mul_mat, ctx.h
    args = [(ctypes.byref(ws[i % copies]), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(ys[i % copies].data_ptr())) for i in range(calls)]

    def run():
        for w, xp, yp in args:
            ctx.check(fn(h, w, xp, 1, yp))

    run()
    ctx.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        run()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (reps * calls)
    nbytes = ws[0].nbytes
    del graph
    for w in ws:
        ctx.free_weight(w)
    return {"K": K, "N": N, "weight_bytes": nbytes, "copies": copies, "calls_per_graph": calls, "us_per_call": us,
            "gbs": nbytes / us / 1e3}


def _product_stack(pkg, ctx, shapes, n_layer, seed):
    """n_layer x the given (type, K, N) products with device-generated weights (Q8_0: N(0, 0.02) quantized on the device;
    K-quants: random valid blocks)."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    layers = []
    for _ in range(n_layer):
        ws = []
        for t, K, N in shapes:
            w = ctx.weight(t, K, N)
            for r0 in range(0, N, 8192):
                rows = min(8192, N - r0)
                blocks = (ctx.quantize_rows(t, torch.randn((rows, K), generator=g, device="cuda") * 0.02) if t == pkg.Q8_0
                          else _random_kquant_blocks(t, rows, K, g))
                ctx.set_weight(w, blocks, offset=r0 * pkg.row_size(t, K))
            ws.append(w)
        layers.append(ws)
    ctx.synchronize()
    return layers


def _time_products(pkg, ctx, stream, layers, M, reps, graph=True):
    """Event-timed passes over every product of the stack with M activation rows (inputs resident, one output
    buffer per shape); returns (ms per pass, weight bytes per pass)."""
    import ctypes

    import torch

    xs, ys, calls = {}, {}, []
    for ws in layers:
        for w in ws:
            if w.ne0 not in xs:
                xs[w.ne0] = torch.randn((M, w.ne0), device="cuda")
            if w.ne1 not in ys:
                ys[w.ne1] = torch.empty((M, w.ne1), device="cuda")
            calls.append((ctypes.byref(w), ctypes.c_void_p(xs[w.ne0].data_ptr()), ctypes.c_void_p(ys[w.ne1].data_ptr())))
    fn, h = ctx.L.b200_mul_mat, ctx.h

    def run():
        for w, x, y in calls:
            ctx.check(fn(h, w, x, M, y))

    run()
    ctx.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            run()
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            if g is not None:
                g.replay()
            else:
                run()
        e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    return ms, sum(w.nbytes for ws in layers for w in ws)


def config4_batched(pkg, ctx, stream, reps=10):
    """Config 4: the Qwen3-TTS 1.7B-shaped talker's products (28 x {q|k|v 2048->4096, o 2048->2048,
    gate|up 2048->12288, down 6144->2048}, Q8_0) for M = 64 concurrent streams: int8 tensor-core products."""
    layers = _product_stack(pkg, ctx, [(pkg.Q8_0, 2048, 4096), (pkg.Q8_0, 2048, 2048), (pkg.Q8_0, 2048, 12288),
                                       (pkg.Q8_0, 6144, 2048)], 28, 41)
    ms, nbytes = _time_products(pkg, ctx, stream, layers, 64, reps)
    ops = 2.0 * 64 * sum(w.ne0 * w.ne1 for ws in layers for w in ws)
    for ws in layers:
        for w in ws:
            ctx.free_weight(w)
    return {"M": 64, "ms_per_step": ms, "tok_s": 64 * 1000.0 / ms, "weight_bytes": nbytes, "gbs": nbytes / ms / 1e6,
            "int8_tops": ops / ms / 1e9}


def config3_prefill(pkg, ctx, stream, reps=2):
    """Config 3's prefill: the Qwen3-ASR 1.7B-shaped decoder's products (28 x {q|k|v 2048->4096, o 2048->2048,
    gate|up 2048->12288 Q4_K; down 6144->2048 Q6_K}) for M = 1500 rows (the head runs on the last row only: one
    2048 -> 151936 Q6_K product, M = 1). K-quant products with many rows run on the int8 tensor cores over an
    int8 expansion of the weights made on the first product (the untimed warm-up pass)."""
    layers = _product_stack(pkg, ctx, [(pkg.Q4_K, 2048, 4096), (pkg.Q4_K, 2048, 2048), (pkg.Q4_K, 2048, 12288),
                                       (pkg.Q6_K, 6144, 2048)], 28, 43)
    head = _product_stack(pkg, ctx, [(pkg.Q6_K, 2048, 151936)], 1, 44)
    ms, nbytes = _time_products(pkg, ctx, stream, layers, 1500, reps, graph=False)
    ms_head, head_bytes = _time_products(pkg, ctx, stream, head, 1, 5)
    ops = 2.0 * 1500 * sum(w.ne0 * w.ne1 for ws in layers for w in ws) + 2.0 * 2048 * 151936
    for ws in layers + head:
        for w in ws:
            ctx.free_weight(w)
    total = ms + ms_head
    return {"M": 1500, "ms": total, "rows_per_s": 1500 * 1000.0 / total, "weight_bytes": nbytes + head_bytes,
            "gbs": (nbytes + head_bytes) / total / 1e6, "int8_tops": ops / total / 1e9,
            "path": "int8 tensor cores (gemm_kq_tc_kernel) over the cached int8 expansion of the K-quant weights"}


def config3_decode(pkg, ctx, stream, steps=128):
    """Config 3's decode phase: 128 batch-1 steps of the Qwen3-ASR 1.7B-shaped decoder (Q4_K attention and gate|up,
    Q6_K down and the 2048 -> 151936 head; random valid blocks), one persistent launch per step."""
    import torch

    dec, c = make_decoder(pkg, ctx, seed=4321, name="asr17")
    x = torch.randn(c["hidden"], generator=torch.Generator(device="cuda").manual_seed(9), device="cuda")
    logits = torch.empty(c["n_vocab"], device="cuda")
    for _ in range(3):
        dec.step_raw(x.data_ptr(), logits.data_ptr())
    ctx.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        dec.step_raw(x.data_ptr(), logits.data_ptr())
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    wb = dec.weight_bytes
    out = {"steps": steps, "ms_per_step": ms, "tok_s": 1000.0 / ms, "weight_bytes": wb, "gbs": wb / ms / 1e6,
           "launches_per_step": dec.launches}
    del dec
    return out


GEMV_CASES = ("q8_0", "q4_k", "q6_k_head_asr17")


def large_gemv(pkg, ctx, stream, reps=20, warmup=3, only=None):
    """Weight GB/s of single large products (matrices far larger than L2), one launch each, CUDA events on the
    context stream: the HBM-bound GEMV kernels without the decode step's dependency chain."""
    import ctypes

    import torch

    out = {}
    cases = [("q8_0", pkg.Q8_0, 4096, 65536), ("q4_k", pkg.Q4_K, 4096, 65536),
             ("q6_k_head_asr17", pkg.Q6_K, 2048, 151936)]
    g = torch.Generator(device="cuda").manual_seed(3)
    for name, t, K, N in cases:
        if only and name != only:
            continue
        w = ctx.weight(t, K, N)
        for r0 in range(0, N, 16384):  # quantize in pieces (device-side, bit-identical to the oracle's quantizer)
            rows = min(16384, N - r0)
            if t == pkg.Q8_0:
                blocks = ctx.quantize_rows(t, torch.randn((rows, K), generator=g, device="cuda") * 0.02)
            else:  # K-quant weights: random valid blocks (uniform bytes, small positive fp16 scales)
                blocks = _random_kquant_blocks(t, rows, K, g)
            ctx.set_weight(w, blocks, offset=r0 * pkg.row_size(t, K))
        x = torch.randn((1, K), generator=g, device="cuda")
        y = torch.empty((1, N), device="cuda")
        ctx.synchronize()
        call = lambda: ctx.check(ctx.L.b200_mul_mat(ctx.h, ctypes.byref(w), ctypes.c_void_p(x.data_ptr()), 1, ctypes.c_void_p(y.data_ptr())))
        for _ in range(warmup):
            call()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            call()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        out[name] = {"K": K, "N": N, "weight_bytes": w.nbytes, "us": ms * 1000.0, "gbs": w.nbytes / ms / 1e6}
        ctx.free_weight(w)
    return out


def _random_kquant_blocks(t, rows, K, g):
    import torch

    bb = {12: 144, 14: 210}[t]
    nb = rows * (K // 256)
    b = torch.randint(0, 256, (nb, bb), generator=g, device="cuda", dtype=torch.int32).to(torch.uint8)
    scale = (torch.rand((nb,), generator=g, device="cuda") * 1e-3 + 1e-4).to(torch.float16).view(torch.uint8).view(nb, 2)
    if t == 12:
        b[:, 0:2] = scale
        b[:, 2:4] = scale
    else:
        b[:, 208:210] = scale
    return b.reshape(-1)


def run_batched(args, pkg, ctx, dist, world, rank, local):
    """Config 4 over N GPUs: the Qwen3-TTS 1.7B-shaped talker's products (28 x {q|k|v 2048->4096, o 2048->2048,
    gate|up 2048->12288, down 6144->2048}, Q8_0) for M = 64 streams, every product split by output rows (rank r holds
    rows [r N/G, (r+1) N/G)) with one all-gather + assembly per product (speech.cpp_b200/column_parallel.py). Inputs
    are resident and replicated; the step is one CUDA graph; strong scaling (the same 64 streams at every N)."""
    import importlib

    import torch

    cp = importlib.import_module(pkg.__name__ + ".column_parallel")
    M, L = 64, 28
    shapes = [(2048, 4096), (2048, 2048), (2048, 12288), (6144, 2048)]
    g = torch.Generator(device="cuda").manual_seed(4000 + rank)
    group = dist.group.WORLD if dist else None
    prods, bufs = [], []
    xs = {K: torch.randn((M, K), generator=g, device="cuda") for K in (2048, 6144)}
    outs = {N: torch.empty((M, N), device="cuda") for _, N in shapes}
    for _ in range(L):
        for K, N in shapes:
            r0, n = cp.row_shard(N, world, rank)
            w = ctx.weight(pkg.Q8_0, K, n)
            for q0 in range(0, n, 4096):
                rows = min(4096, n - q0)
                ctx.set_weight(w, ctx.quantize_rows(pkg.Q8_0, torch.randn((rows, K), generator=g, device="cuda") * 0.02),
                               offset=q0 * pkg.row_size(pkg.Q8_0, K))
            prods.append((cp.ColumnParallelProduct(lambda w, x, out: ctx.mul_mat(w, x, out=out), w, N, group=group), K, N))
            bufs.append((torch.empty((M, n), device="cuda"), torch.empty((world, M, n), device="cuda")))
    ctx.synchronize()
    stream = ctx.torch_stream()

    def step():
        for (prod, K, N), (lo, ga) in zip(prods, bufs):
            prod(xs[K], lo, ga, outs[N])

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    steps = args.steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(steps):
                graph.replay()
            ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph
    torch.cuda.synchronize()
    ms_step = ms / steps
    wbytes = sum(p[0].w.nbytes for p in prods)
    for p in prods:
        ctx.free_weight(p[0].w)
    peak, peak_kind = peaks()
    achieved = wbytes / (ms_step / 1000.0) / 1e9
    return {
        "metric": "batched decode tok/s, Qwen3-TTS 1.7B-shaped talker products (Q8_0, M = 64 streams)", "value": M * 1000.0 / ms_step,
        "unit": UNIT, "n_gpus": world, "steps": steps, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "dtype": "int8xint8->int32, f32 accumulate", "data": "synthetic",
        "config": {"workload": "config 4: 28 x {q|k|v 2048->4096, o 2048->2048, gate|up 2048->12288, down 6144->2048}, Q8_0, M = 64",
                   "global_batch": M, "parallelism": f"column split x{world} (all-gather per product)" if world > 1 else "single",
                   "l2": f"weights {wbytes / 1e9:.2f} GB per GPU > 126 MB L2"},
        "roofline": {"bound": "hbm", "kernel": "the product stack (tensor-core GEMMs + all-gathers)", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "algorithmic_bytes_per_step": wbytes, "traffic": None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6650"},
        "gpu_launches": 2 * L * len(shapes) * steps, "clocks": clk.summary(),
    }


def int8_peak_tops(seconds=1.0):
    """Dense int8 tensor throughput of this GPU, measured with the library GEMM (torch._int_mm, cuBLASLt) on
    8192^3 int8 x int8 -> int32, best of repeated launches: the denominator of the int8 roofline (like the measured
    cuBLAS bf16 figure for bf16). None if the library path is unavailable."""
    import torch

    try:
        n = 8192
        a = torch.randint(-64, 64, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-64, 64, (n, n), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best, t_end = None, time.perf_counter() + seconds
        while time.perf_counter() < t_end or best is None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                torch._int_mm(a, b)
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1) / 5
            best = ms if best is None or ms < best else best
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except Exception:
        return None


def run_prefill(args, pkg, ctx, dist, world, rank, local):
    """Config 3's prefill as its own line: M = 1500 rows through the Qwen3-ASR 1.7B-shaped product stack (Q4_K / Q6_K)
    plus the head on the last row. Single stream per GPU: with N > 1, N independent replicas."""
    import torch

    stream = ctx.torch_stream()
    if dist:
        dist.barrier()
    with Clocks(local) as clk:
        r = config3_prefill(pkg, ctx, stream, reps=max(2, args.steps // 5))
    ms = r["ms"]
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ipeak = int8_peak_tops()
    ipeak_src = "measured: torch._int_mm (cuBLASLt) int8 8192^3, best of 5-launch means over 1 s" if ipeak else None
    if not ipeak:
        ipeak, ipeak_src = 4500.0, "nominal dense int8 (the library int8 GEMM was unavailable)"
    return {
        "metric": "prefill rows/s, Qwen3-ASR 1.7B-shaped decoder products (Q4_K / Q6_K), M = 1500", "value": world * 1500 * 1000.0 / ms,
        "unit": "rows/s", "n_gpus": world, "steps": max(2, args.steps // 5), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "dtype": "int8xint8->int32, f32 accumulate", "data": "synthetic",
        "config": {"workload": "config 3 prefill: 28 x {q|k|v 2048->4096, o 2048->2048, gate|up 2048->12288 Q4_K, down 6144->2048 Q6_K}"
                               " x 1500 rows + head 2048->151936 Q6_K x 1 row", "global_batch": 1500 * world,
                   "parallelism": f"replicas x{world}" if world > 1 else "single"},
        "roofline": {"bound": "tensor", "kernel": "gemm_kq_tc_kernel", "achieved": r["int8_tops"], "unit": "TOP/s int8",
                     "peak": ipeak, "frac": r["int8_tops"] / ipeak, "peak_source": ipeak_src, "traffic": None},
        "clocks": clk.summary(), "gpu_launches": (28 * 4 * 2 + 1) * max(2, args.steps // 5),
    }


def side_configs(args, pkg, ctx):
    """BASELINE.json's other configurations at one GPU, each with its roofline fraction."""
    stream = ctx.torch_stream()
    peak, kind = peaks()
    out = {"c2_tts06_decode": config2_decode(pkg, ctx, stream, steps=max(args.steps, 100), warmup=args.warmup)}
    r = config1_gemv(pkg, ctx, stream)
    out["c1_gemv_q8_0"] = dict(r, frac=r["gbs"] / peak, bound="hbm", **peak_fields(peak, kind))
    r = config3_decode(pkg, ctx, stream)
    out["c3_asr17_decode"] = dict(r, frac=r["gbs"] / peak, bound="hbm", **peak_fields(peak, kind))
    r = config3_prefill(pkg, ctx, stream)
    ipeak, isrc = int8_peak_or_nominal()
    out["c3_asr17_prefill"] = dict(r, bound="int8 tensor", frac=r["int8_tops"] / ipeak, peak=ipeak, peak_unit="TOP/s int8", peak_source=isrc,
                                   hbm_frac=r["gbs"] / peak)
    r = config4_batched(pkg, ctx, stream)
    out["c4_batched_m64"] = dict(r, frac=r["gbs"] / peak, bound="hbm", int8_frac=r["int8_tops"] / ipeak, **peak_fields(peak, kind))
    out["gemv_large"] = {k: dict(v, frac=v["gbs"] / peak) for k, v in large_gemv(pkg, ctx, stream).items()}
    return out


def int8_peak_or_nominal():
    ipeak = int8_peak_tops()
    if ipeak:
        return ipeak, "measured: torch._int_mm (cuBLASLt) int8 8192^3, best of 5-launch means over 1 s"
    return 4500.0, "nominal dense int8 (the library int8 GEMM was unavailable)"


def run_b200(args):
    import torch

    world, rank, local = dist_setup()
    dist = None
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    pkg = load_package()
    ctx = pkg.Context(local)
    if args.workload == "gemv":
        # one large single-column product (profiling and tuning of the HBM-bound GEMV kernel): --steps timed launches
        # after --warmup untimed ones
        r = large_gemv(pkg, ctx, ctx.torch_stream(), reps=max(args.steps, 1), warmup=args.warmup, only=args.gemv_case)
        peak, kind = peaks()
        v = r[args.gemv_case]
        emit({"metric": "weight GB/s of one large single-column product (TMA GEMV)", "value": v["gbs"], "unit": "GB/s",
              "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": v["us"] / 1000.0,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x q8",
              "data": "synthetic", "config": {"workload": f"single product {args.gemv_case}", "K": v["K"], "N": v["N"],
                                              "l2": "weights > 126 MB L2"},
              "roofline": dict({"bound": "hbm", "achieved": v["gbs"], "unit": "GB/s", "frac": v["gbs"] / peak}, **peak_fields(peak, kind))})
        ctx.close()
        return 0
    if args.workload == "decode":
        r = config2_decode(pkg, ctx, ctx.torch_stream(), steps=args.steps, warmup=args.warmup, seed=1234 + rank)
        ctx.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            emit({"metric": "decode tok/s, Qwen3-TTS 0.6B talker decode-step matmul stack (Q8_0, batch 1)", "value": r["tok_s"],
                  "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                  "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->int32, f32 accumulate",
                  "data": "synthetic", "config": {"workload": r["workload"], "global_batch": 1, "seq_len": 1, "parallelism": "single"},
                  "roofline": {k: r[k] for k in ("bound", "kernel", "frac", "peak", "peak_source", "traffic", "traffic_source")} | {
                      "achieved": r["gbs"], "unit": "GB/s"},
                  "e2e": {"value": r["e2e_tok_s"], "unit": UNIT, "h2d_bytes_per_step": r["e2e_h2d_bytes_per_step"],
                          "d2h_bytes_per_step": r["e2e_d2h_bytes_per_step"]}, "gpu_launches": r["launches_per_step"] * args.steps})
        return 0
    if args.workload in ("batched", "prefill"):
        res = {"batched": run_batched, "prefill": run_prefill}[args.workload](args, pkg, ctx, dist, world, rank, local)
        ctx.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            res.update(warmup=args.warmup, vs_baseline=None)
            emit(res)
        return 0

    # ---- the headline: config 5 ----
    res, keep = run_moe(args, pkg, ctx, dist, world, rank, local)
    if dist:
        dist.barrier()
    if rank == 0 and world == 1 and not args.no_cpu:
        # the CPU-baseline leg: the oracle's stack timed on this host, and the parity check of layer 0 on the same
        # weights and inputs as the GPU's
        nthreads = host_threads()
        res["parity"] = moe_parity(pkg, ctx, keep["weights"][0], keep["weights"][args.moe_layers], keep["x0"], keep["ids0"], keep["w0"],
                                   keep["y0"], nthreads)
        v, sample, _ = cpu_moe_rate(MOE, args.ref_tokens, nthreads, 1, 3)
        res["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": nthreads, "kind": "port", "sample": sample}
    for w in keep["weights"]:
        ctx.free_weight(w)
    if rank == 0 and world == 1 and not args.no_configs:
        res["configs"] = side_configs(args, pkg, ctx)
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(res)
    return 0


class _StdoutToStderr:
    """Points file descriptor 1 at stderr until restore(): libraries (NCCL's version banner, warnings) write to stdout,
    and the driver reads rank 0's stdout for the one JSON line."""

    def __init__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)

    def restore(self):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


def emit(line):
    """Prints the result line on the real stdout."""
    if _QUIET is not None:
        _QUIET.restore()
    print(json.dumps(line), flush=True)


_QUIET = None


def main():
    global _QUIET
    _QUIET = _StdoutToStderr()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline and parity leg")
    ap.add_argument("--no-configs", action="store_true", help="skip the side measurements of configs 1-4")
    ap.add_argument("--workload", default="moe", choices=["moe", "decode", "batched", "prefill", "gemv"],
                    help="moe: config 5, expert-parallel (the headline line); decode: config 2's decode step alone; batched: "
                         "config 4, column-split; prefill: config 3's prefill; gemv: one large single-column product")
    ap.add_argument("--gemv-case", default="q8_0", choices=list(GEMV_CASES), help="product of --workload gemv")
    ap.add_argument("--moe-layers", type=int, default=48, help="MoE layers per step (48 = config 5; fewer only for profiling)")
    ap.add_argument("--moe-combine", default="nccl", choices=["peer", "nccl"],
                    help="N > 1: how the ranks' partial sums are added: an NCCL all-reduce, or the combine kernel over NVLink peer memory")
    ap.add_argument("--ref-tokens", type=int, default=32, help="tokens of the 256 the CPU legs run through the 48 layers")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
