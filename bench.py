"""Qwen3-8B decode throughput on B200 (the reference's headline metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one step = one decode step of the executor): Qwen3-8B architecture (36 layers,
hidden 4096, 32 q / 8 kv heads, head_dim 128, intermediate 12288, vocab 151936), random-init
bf16 weights N(0, 0.02) (norm gains 1), batch 128, context 2048 per request = a 1024-token
prefix held once in the pool (64 pages referenced by every page table, as a radix-cache match
would) + 1024 unique tokens, page size 16, page placement shuffled over the pool (seed 3).
KV contents are synthetic N(0, 1) bf16 (no prefill is timed). Every step reads ~35 GB
(weights 16.4 GB + unique KV 19.5 GB), far above the 126 MB L2, so no flush is needed.

value  : 128 tokens / step time, the step replayed as a CUDA graph on device-resident inputs
         (CUDA events on the launching stream, max over ranks).
e2e    : the same steps through msgl_model_step_host: pinned host batch -> H2D -> graph ->
         D2H of the 128 next tokens -> stream sync, all inside the timed region.
roofline: the paged decode-attention kernel (the largest share of the step) timed alone on the
         same stream over all 36 layers' pools: unique KV bytes per launch / mean duration,
         against MEASURED_PEAKS.json hbm_gbs.
cpu_baseline: the reference's own CPU code (oracle/_ref: Linear::forward of the 4 layer
         projections + lm_head; attention from the C restatement, as the reference has no
         paged/GQA attention) on a bounded token sample, extrapolated to the full step.
N > 1: tensor parallelism over the N GPUs (one process each, NCCL over NVLink): the same
         128-request step, heads / FFN columns / vocab rows sharded (strong scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mini-sglang-cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402

METRIC = "Qwen3-8B decode tok/s (batch 128, ctx 2048, 1024-token shared prefix)"
UNIT = "tokens/s"
CFG8B = dict(num_layers=36, hidden=4096, num_q_heads=32, num_kv_heads=8, head_dim=128,
             inter=12288, vocab=151936, eps=1e-6, rope_base=1e6, max_position=4096)
BATCH, CTX, PREFIX, PAGE = 128, 2048, 1024, 16
# host threads of the CPU reference (fixed, so the baseline does not follow the host's core count)
CPU_THREADS = 16


def workload_config(n_gpus):
    return {"workload": "qwen3-8b-decode", "model_arch": "Qwen3-8B", "global_batch": BATCH,
            "batch_per_gpu": BATCH, "seq_len": CTX, "shared_prefix": PREFIX, "page_size": PAGE,
            "parallelism": f"tp{n_gpus}" if n_gpus > 1 else "tp1",
            "l2": "inputs larger than L2 (35 GB read per step)"}


# ------------------------------------------------------------------------------ page tables
def build_pages(seed=3):
    """Page tables for the 128 requests: 64 shared prefix pages + 64 unique pages each,
    drawn LIFO (KVCachePool order) from a free list shuffled with `seed`."""
    from msgl.model import PagePool
    n_prefix, n_own = PREFIX // PAGE, (CTX - PREFIX) // PAGE
    num_pages = n_prefix + BATCH * n_own + 16
    pool = PagePool(num_pages)
    rng = np.random.default_rng(seed)
    rng.shuffle(pool.free)
    prefix = [pool.allocate() for _ in range(n_prefix)]
    pt = np.zeros((BATCH, n_prefix + n_own), np.int32)
    for r in range(BATCH):
        pt[r] = prefix + [pool.allocate() for _ in range(n_own)]
    return num_pages, pt


def decode_batch_host(pt, vocab, seed=1):
    rng = np.random.default_rng(seed)
    pos = np.full(BATCH, CTX - 1, np.int32)
    slots = (pt[:, (CTX - 1) // PAGE] * PAGE + (CTX - 1) % PAGE).astype(np.int32)
    return dict(input_ids=rng.integers(0, vocab, BATCH).astype(np.int32), positions=pos,
                slot_mapping=slots, page_table=np.ascontiguousarray(pt),
                seq_lens=np.full(BATCH, CTX, np.int32),
                q_indptr=np.arange(BATCH + 1, dtype=np.int32),
                last_idx=np.arange(BATCH, dtype=np.int32))


# ------------------------------------------------------------------------------ clocks
# DRAM bytes (read + write) of one paged_decode_cascade_kernel launch at this workload (8 kv
# heads), from one ncu capture of `bench.py --case attention_cascade` (547 404 544 B read +
# 11 156 224 B written; the algorithmic unique K+V bytes are 541 065 216 B).
PAGED_DECODE_TRAFFIC_BYTES = 558_560_768


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of this rank's GPU during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu, self.p, self.out = str(gpu_index), None, ""
        try:  # nvidia-smi numbers GPUs independently of CUDA_VISIBLE_DEVICES: use the PCI id
            import torch
            pr = torch.cuda.get_device_properties(gpu_index)
            self.gpu = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
        except Exception:
            pass

    def __enter__(self):
        self.first = ""
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        if self.p:  # the timed region starts once the sampler is producing samples
            import select
            r, _, _ = select.select([self.p.stdout], [], [], 10.0)
            if r:
                self.first = self.p.stdout.readline()
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                rest, _ = self.p.communicate(timeout=5)
                self.out = self.first + (rest or "")
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.out = self.first

    def summary(self):
        sm, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------ CPU reference
class CpuModelRef:
    """A step of the model on the reference CPU code, timed on a bounded sample.

    Each worker thread carries one token through one decoder layer: the layer's projections by
    the reference's Linear::forward on persistent weights (as in a loaded model) -- qkv, o_proj,
    and gate_up + down (dense) or the router and top_k experts' gate_up + down (MoE, the expert
    loop of qwen3_moe.cpp:62-111) -- plus one request's attention over `ctx` tokens (the C
    restatement: the reference has no paged / GQA attention). Another sample carries one token
    through lm_head. `threads` tokens therefore advance one layer per sample and a step of
    `tokens` tokens through `layers` layers (+ `lm_rows` lm_head rows) extrapolates linearly."""

    def __init__(self, cfg, ctx, threads=None):
        from oracle import Oracle, RefLib
        self.ref, self.orc = RefLib(), Oracle()
        t = threads or min(CPU_THREADS, os.cpu_count() or 1)
        self.threads = max(1, t)
        self.cfg, self.ctx = cfg, int(ctx)
        H, V, D = cfg["hidden"], cfg["vocab"], 128
        hq, hkv = cfg["num_q_heads"], cfg["num_kv_heads"]
        E, k, Im = cfg.get("num_experts", 0), cfg.get("top_k", 0), cfg.get("moe_inter", 0)
        L = self.ref.lib
        shapes = [((hq + 2 * hkv) * D, H), (H, hq * D)]
        if E:  # router, then top_k distinct experts (a token's route)
            shapes += [(E, H)] + [(2 * Im, H), (H, Im)] * k
        else:
            shapes += [(2 * cfg["inter"], H), (H, cfg["inter"])]
        self.handles = []
        for n, kk in shapes:
            w = np.full((n, kk), 0.01, np.float32)  # values do not change fp32 loop timing
            self.handles.append((L.ref_linear_create(w.ctypes.data, kk, n), n, kk))
        wl = np.full((V, H), 0.01, np.float32)
        self.lm = L.ref_linear_create(wl.ctypes.data, H, V)
        ctx_pages = -(-self.ctx // PAGE)
        rng = np.random.default_rng(0)
        self.kp = rng.standard_normal((ctx_pages * PAGE, hkv * D)).astype(np.float32)
        self.vp = rng.standard_normal((ctx_pages * PAGE, hkv * D)).astype(np.float32)
        self.pt = np.arange(ctx_pages, dtype=np.int32)[None, :]

    def close(self):
        L = self.ref.lib
        for h, _, _ in self.handles:
            L.ref_linear_destroy(h)
        L.ref_linear_destroy(self.lm)
        self.handles = []

    def _timed(self, fn):
        ts = [threading.Thread(target=fn) for _ in range(self.threads)]
        t0 = time.perf_counter()
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        return time.perf_counter() - t0

    def _timed_pair(self):
        """Wall seconds of one layer sample and of one lm_head sample (threads tokens each)."""
        return self._last

    def sample(self, tokens, lm_rows, layers):
        """(tokens per second of the full step, description of the sample)."""
        cfg = self.cfg
        H, V, D = cfg["hidden"], cfg["vocab"], 128
        hq, hkv = cfg["num_q_heads"], cfg["num_kv_heads"]
        L = self.ref.lib

        def layer_worker():
            for h, n, k in self.handles:
                xin = np.full((1, k), 0.1, np.float32)
                out = np.empty((1, n), np.float32)
                L.ref_linear_run(h, xin.ctypes.data, 1, out.ctypes.data)
            q = np.full((1, hq * D), 0.01, np.float32)
            self.orc.paged_attention(q, self.kp, self.vp, self.pt, [self.ctx], [0, 1], hq, hkv, D,
                                     PAGE)

        def lm_worker():
            xin = np.full((1, H), 0.1, np.float32)
            out = np.empty((1, V), np.float32)
            L.ref_linear_run(self.lm, xin.ctypes.data, 1, out.ctypes.data)

        w_layer = self._timed(layer_worker)
        w_lm = self._timed(lm_worker)
        self._last = (w_layer, w_lm)
        step_s = (tokens * layers * w_layer + lm_rows * w_lm) / self.threads
        desc = (f"{self.threads} tokens x 1 of {layers} layers (projections by the reference "
                f"Linear::forward{', MoE expert loop' if cfg.get('num_experts') else ''}; "
                f"attention over {self.ctx} tokens, C restatement) + {self.threads} tokens x "
                f"lm_head, extrapolated to {tokens} tokens x {layers} layers + {lm_rows} lm_head "
                f"rows; fp32")
        return tokens / step_s, desc


class CpuReference(CpuModelRef):
    """The Qwen3-8B decode step (128 tokens, context 2048) on the reference CPU code."""

    def __init__(self, threads=None):
        super().__init__(CFG8B, CTX, threads)

    def sample(self, layers=36):
        return super().sample(BATCH, BATCH, layers)


def reference_workload(name):
    """(metric, value, sample, config) of a non-default workload on the reference CPU code: the
    same sample as that workload's cpu_baseline."""
    if name == "qwen3-0.6b-greedy":
        cpu = CpuModelRef(dict(CFG06B, max_position=512), 144)
        _, sample = cpu.sample(1, 1, 1)
        w_layer, w_lm = cpu._timed_pair()
        run_s = ((4 * 128 + 4 * 31) * 28 * w_layer + 4 * 32 * w_lm) / cpu.threads
        cpu.close()
        return ("Qwen3-0.6B greedy generation tok/s (4 x 128-token prompts, 32 new tokens each)",
                128 / run_s, sample, cpu.threads, {"workload": name, "model_arch": "Qwen3-0.6B"})
    if name == "qwen3-0.6b-decode-ragged":
        ctx = np.random.default_rng(2).integers(512, 4097, 64)
        cpu = CpuModelRef(CFG06B, int(ctx.mean()))
        v, sample = cpu.sample(64, 64, 28)
        cpu.close()
        return ("Qwen3-0.6B decode tok/s (batch 64, ctx U[512,4096], permuted pages)", v, sample,
                cpu.threads, {"workload": name, "model_arch": "Qwen3-0.6B", "global_batch": 64})
    if name == "qwen3-32b-mixed":
        dctx = np.random.default_rng(2).integers(1024, 8193, 96)
        cpu = CpuModelRef(CFG32B, int(dctx.mean()))
        v, sample = cpu.sample(2144, 97, 64)
        cpu.close()
        return ("Qwen3-32B mixed chunked-prefill tok/s (2048-token chunk + 96 decodes per step)",
                v, sample, cpu.threads, {"workload": name, "model_arch": "Qwen3-32B"})
    cpu = CpuModelRef(CFG30BA3B, 1024)
    v, sample = cpu.sample(256, 256, 48)
    cpu.close()
    return ("Qwen3-30B-A3B decode tok/s (batch 256, ctx 1024)", v, sample, cpu.threads,
            {"workload": name, "model_arch": "Qwen3-30B-A3B", "global_batch": 256})


def run_reference_arm(args, rank):
    if rank != 0:
        return 0
    if args.workload != "qwen3-8b-decode":
        vals = []
        for i in range(args.warmup + args.steps):
            metric, v, sample, cores, cfg = reference_workload(args.workload)
            if i >= args.warmup:
                vals.append(v)
        value = float(np.median(vals))
        print(json.dumps({"impl": "reference", "metric": metric, "value": value, "unit": UNIT,
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "extrapolated": True, "higher_is_better": True, "scaling": "strong",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
                          "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores,
                                           "kind": "reference", "sample": sample,
                                           "extrapolated": True},
                          "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    cpu = CpuReference()
    vals = []
    for i in range(args.warmup + args.steps):
        v, sample = cpu.sample()
        if i >= args.warmup:
            vals.append(v)
    cpu.close()
    cores = cpu.threads
    value = float(np.median(vals))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * BATCH / value, "extrapolated": True,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "reference",
                             "sample": sample, "extrapolated": True},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ timing
def timed_blocks(fn, args, world, dev, stream, barrier, max_over_ranks):
    """`args.blocks` back-to-back blocks of exactly `args.steps` steps, each bracketed by a barrier
    and a device synchronise; returns each block's ms per step (max over ranks). Before each
    block the ranks meet on the device (a one-element NCCL all-reduce on the timing stream), so
    the start event fires on every rank once all ranks have arrived: launch skew between ranks
    stays outside the timed region."""
    import torch
    import torch.distributed as dist
    out = []
    for _ in range(args.blocks):
        barrier()
        torch.cuda.synchronize()
        if world > 1:
            dist.all_reduce(torch.zeros(1, device=dev))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        out.append(max_over_ranks(e0.elapsed_time(e1) / args.steps))
    return out


# ------------------------------------------------------------------------------ parity record
PARITY_CFG = dict(num_layers=3, hidden=512, num_q_heads=8, num_kv_heads=2, head_dim=128, inter=768,
                  vocab=1000, eps=1e-6, rope_base=1e6, max_position=512, page_size=16)


def parity_case(rank, world, dev):
    """The executor at this run's tensor-parallel size on a small Qwen3 (3 layers, hidden 512,
    8 q / 2 kv heads, head_dim 128, vocab 1000; weights N(0, 0.05) from the device generator,
    norm gains 1): prefill of 3 requests (5, 20, 33 tokens) + 3 greedy decode steps, on its own
    communicator. Rank 0 compares every step's all-gathered logits with the oracle; every rank's
    logits must be the same bits. Returns the record printed in the bench line."""
    import hashlib

    import torch
    import torch.distributed as dist

    from msgl import ops
    from msgl.model import BatchBuilder, PagePool, Qwen3Model, Request, TPComm
    cfg = PARITY_CFG
    H, D, hq, hkv, I, V = 512, 128, 8, 2, 768, 1000
    names = [("embed", (V, H))]
    for l in range(cfg["num_layers"]):
        p = f"layers.{l}."
        names += [(p + "input_ln", (H,)), (p + "qkv", ((hq + 2 * hkv) * D, H)), (p + "q_norm", (D,)),
                  (p + "k_norm", (D,)), (p + "o", (H, hq * D)), (p + "post_ln", (H,)),
                  (p + "gate_up", (2 * I, H)), (p + "down", (H, I))]
    names += [("norm", (H,)), ("lm_head", (V, H))]
    comm = None
    if world > 1:
        uid = [TPComm.new_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = TPComm(rank, world, uid[0])
    model = Qwen3Model(cfg, max_tokens=128, max_reqs=4, tp_rank=rank, tp_size=world)
    wts = {}
    for i, (n, shape) in enumerate(names):
        if len(shape) == 1:
            bits = np.full(shape, 0x3F80, np.uint16)
        else:
            t = ops.fill_normal_(torch.empty(shape, dtype=torch.bfloat16, device=dev), seed=11,
                                 stream_id=i, std=0.05)
            bits = t.view(torch.int16).cpu().numpy().view(np.uint16)
        model.set_weight_bits(n, bits)
        wts[n] = bits
    if comm is not None:
        model.set_tp(comm)
    model.alloc_kv(32)
    orc = None
    if rank == 0:
        from oracle import Oracle, OracleModel, from_bf16_bits
        orc = OracleModel(Oracle(), cfg, {k: from_bf16_bits(v).reshape(v.shape) for k, v in wts.items()},
                          num_slots=32 * 16)
    rng = np.random.default_rng(1)
    reqs = [Request(list(rng.integers(0, V, n))) for n in (5, 20, 33)]
    bb = BatchBuilder(PagePool(32))
    worst, agree, total, clear_ok, digests = 0.0, 0, 0, True, []
    for step in range(4):
        sb = bb.build(reqs, decode=step > 0, device=dev, max_pages=4)
        nxt, lg = model.forward(sb, logits=True)
        torch.cuda.synchronize()
        got, ids = lg.cpu().numpy(), nxt.cpu().numpy()
        digests.append(hashlib.sha1(got.tobytes() + ids.tobytes()).hexdigest())
        if orc is not None:
            h = {k: v.cpu().numpy() for k, v in sb.tensors.items()}
            ref = orc.forward(h["input_ids"], h["positions"], h["slot_mapping"], h["page_table"],
                              h["seq_lens"], h["q_indptr"])
            worst = max(worst, float(np.linalg.norm(got - ref) / np.linalg.norm(ref)))
            top2 = np.sort(ref, axis=1)[:, -2:]
            clear = (top2[:, 1] - top2[:, 0]) > 4 * float(np.abs(got - ref).max())
            clear_ok &= bool(np.array_equal(ids[clear], ref.argmax(axis=1)[clear]))
            agree += int((ids == ref.argmax(axis=1)).sum())
            total += ids.size
        for r, t in zip(reqs, ids):
            r.cached_len = r.device_len
            r.input_ids.append(int(t))
    same = True
    if world > 1:
        allg = [None] * world
        dist.all_gather_object(allg, digests)
        same = all(a == allg[0] for a in allg)
    err = ops.device_error()
    del model
    if comm is not None:
        comm.close()
    return {"case": f"qwen3 3 layers h512 8/2 heads vocab 1000, tp{world}, prefill + 3 decode "
                    "steps vs the fp32 oracle", "max_rel_l2": worst, "tol": 2e-2,
            "ids_equal": f"{agree}/{total}", "margin_clear_ids_equal": clear_ok,
            "ranks_identical": same,
            "pass": bool(worst < 2e-2 and clear_ok and same and err == (0, 0))}


# ------------------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local_rank):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import msgl
    from msgl import ops
    from msgl.model import (SHARED_PREFIX_DETECT, BatchT, Qwen3Model, TPComm, device_view,
                            make_step, shard_plan)

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    msgl.lib()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    parity = parity_case(rank, world, dev)

    # tensor parallel over the `world` GPUs: every rank runs the same 128-request step on its
    # shard (heads / FFN columns / vocab rows); NCCL id from rank 0 through the process group
    comm = None
    if world > 1:
        uid = [TPComm.new_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = TPComm(rank, world, uid[0])
    plan = shard_plan(CFG8B["num_q_heads"], CFG8B["num_kv_heads"], CFG8B["inter"],
                      CFG8B["vocab"], rank, world)
    hq_l, hkv_l = plan["q_heads"], plan["kv_heads"]

    num_pages, pt = build_pages()
    model = Qwen3Model(CFG8B, max_tokens=BATCH, max_reqs=BATCH, tp_rank=rank, tp_size=world)
    if comm is not None:
        model.set_tp(comm)
    model.random_init(seed=0, std=0.02)
    model.alloc_kv(num_pages)
    L = CFG8B["num_layers"]
    pools = [model.kv_pool(l) for l in range(L)]
    for l, (k, v, n) in enumerate(pools):  # synthetic KV contents, N(0,1)
        for j, p in enumerate((k, v)):
            t = device_view(p, (n * hkv_l * 128,), torch.bfloat16)
            ops.fill_normal_(t, seed=4, stream_id=2 * l + j, std=1.0)
    host = decode_batch_host(pt, CFG8B["vocab"])
    sb = make_step(host, True, dev, CTX, 1)
    nxt = torch.empty(BATCH, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    lib = msgl.lib()
    sp = stream.cuda_stream
    # kernels of ours per step, counted on one eager step (graph replays launch nothing from the
    # host, so the count is taken outside them)
    n0 = lib.msgl_kernel_launches()
    model.forward(sb, out=nxt)
    launches_per_step = lib.msgl_kernel_launches() - n0
    torch.cuda.synchronize()

    # ---- value: device-resident inputs, graph replay; several blocks of `steps` steps
    for _ in range(max(args.warmup, 3)):
        model.forward(sb, out=nxt, graph=True)
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        blocks = timed_blocks(lambda: model.forward(sb, out=nxt, graph=True), args, world, dev,
                              stream, barrier, max_over_ranks)
    ms = float(np.median(blocks))
    err = ops.device_error()
    assert err == (0, 0), f"device error word {err}"

    # ---- e2e: host buffers through msgl_model_step_host
    pinned = {k: torch.from_numpy(v).pin_memory() for k, v in host.items()}
    hb = BatchT(BATCH, BATCH, 1, pt.shape[1], CTX, 1,
                *[pinned[k].data_ptr() for k in ("input_ids", "positions", "slot_mapping",
                                                  "page_table", "seq_lens", "q_indptr",
                                                  "last_idx")], SHARED_PREFIX_DETECT)
    out_host = torch.empty(BATCH, dtype=torch.int32).pin_memory()
    step_host = lambda: msgl.check(lib.msgl_model_step_host(model.h, C.addressof(hb),
                                                            out_host.data_ptr(), 1, sp))
    for _ in range(max(args.warmup, 3)):
        step_host()
    blocks_e2e = timed_blocks(step_host, args, world, dev, stream, barrier, max_over_ranks)
    ms_e2e = float(np.median(blocks_e2e))
    h2d = sum(v.nbytes for v in host.values())
    d2h = BATCH * 4
    assert torch.equal(out_host.to(dev), nxt), "host step and device step disagree"

    # ---- roofline: the step's decode attention alone, every layer's pool (the cascade over the
    # shared prefix; with one kv head per rank the executor runs the plain kernel instead)
    hq, hkv = hq_l, hkv_l  # this rank's heads
    q = torch.empty(BATCH, hq, 128, dtype=torch.bfloat16, device=dev)
    ops.fill_normal_(q, seed=5, std=1.0)
    aout = torch.empty_like(q)
    shared = int(sb.struct.shared_prefix_pages)
    assert shared == PREFIX // PAGE, shared
    wsn = lib.msgl_paged_attention_cascade_workspace_size(BATCH, CTX, shared, hq, hkv, 128)
    ws = torch.zeros(wsn, dtype=torch.uint8, device=dev)
    pt_d, seq_d = sb.tensors["page_table"], sb.tensors["seq_lens"]

    cascade = hkv % 4 == 0  # the executor's rule (engine/layers.h, Attention::forward)
    if not cascade:
        ws = ops.attention_workspace(BATCH, CTX, hq, hkv, dev)

    def attn(l):
        k, v, n = pools[l]
        if cascade:
            msgl.check(lib.msgl_paged_attention_decode_cascade(
                q.data_ptr(), k, v, n, pt_d.data_ptr(), pt_d.shape[1], seq_d.data_ptr(), BATCH,
                CTX, shared, hq, hkv, 128, PAGE, 1.0 / 128 ** 0.5, aout.data_ptr(), ws.data_ptr(),
                ws.numel(), sp))
        else:
            msgl.check(lib.msgl_paged_attention_decode(
                q.data_ptr(), k, v, n, pt_d.data_ptr(), pt_d.shape[1], seq_d.data_ptr(), BATCH,
                CTX, hq, hkv, 128, PAGE, 1.0 / 128 ** 0.5, aout.data_ptr(), ws.data_ptr(),
                ws.numel(), sp))

    for l in range(L):
        attn(l)
    torch.cuda.synchronize()
    reps = 3
    e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e4.record(stream)
    for _ in range(reps):
        for l in range(L):
            attn(l)
    e5.record(stream)
    torch.cuda.synchronize()
    attn_ms = e4.elapsed_time(e5) / (reps * L)
    kv_row = hkv * 128 * 2 * 2  # K and V bytes per token
    unique_bytes = (PREFIX + BATCH * (CTX - PREFIX)) * kv_row
    per_request_bytes = BATCH * CTX * kv_row
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = unique_bytes / (attn_ms * 1e-3) / 1e9

    if rank == 0:
        cpu = CpuReference()
        cpu.sample()
        cpu_val, sample = cpu.sample()
        cpu.close()
        cores = cpu.threads
        line = {
            "metric": METRIC, "value": BATCH / (ms * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "blocks_ms_per_step": [round(b, 4) for b in blocks],
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, N(0,1) KV, random token ids)",
            "config": workload_config(world),
            "e2e": {"value": BATCH / (ms_e2e * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e, "blocks_ms_per_step": [round(b, 4) for b in blocks_e2e]},
            "roofline": {"kernel": "paged_decode_cascade_kernel" if cascade else "paged_decode_kernel",
                         "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         # the capture is of 8 kv heads; a TP rank reads its own heads only
                         "traffic": (PAGED_DECODE_TRAFFIC_BYTES * hkv // CFG8B["num_kv_heads"])
                                    if cascade else None,
                         "algorithmic_bytes_per_launch": unique_bytes,
                         "per_request_bytes_per_launch": per_request_bytes,
                         "launch_ms": attn_ms,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": {"value": cpu_val, "unit": UNIT, "cores": cores, "kind": "reference",
                             "sample": sample},
            "clocks": clk.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_per_step": launches_per_step,
            "parity": parity,
            "weights_gb": model.weight_bytes() / 1e9,
        }
        print(json.dumps(line), flush=True)
    # graphs holding NCCL calls and the communicator go before the process group
    del model
    if comm is not None:
        comm.close()
    return 0


def run_case(args):
    """Small single-kernel cases at the bench's shapes, for profiling (one layer, < 1 GB):
    `attention` / `attention_cascade`: paged decode attention (plain / cascade over the shared
    prefix), 128 requests x 2048 context (shared 1024 prefix);
    `gemm`: the gate_up + SwiGLU projection of one layer at 128 tokens (201 MB of weights);
    `gemm_qkv`: the qkv projection at 128 tokens; `gemm_partials`: o_proj at 128 tokens as
    split-K partials; `gemm_prefill`: gate_up + SwiGLU at 2048 tokens; `attention_ragged`: the
    plain decode of the Qwen3-0.6B ragged step (64 requests, contexts U[512, 4096], permuted
    pages, 16 q / 8 kv heads, ~0.6 GB of KV); `moe_gate_up`: the Qwen3-30B-A3B experts' grouped
    gate_up + SwiGLU at 256 decode tokens x top-8 (128 experts x 1536 x 2048, 0.8 GB)."""
    import torch

    import msgl
    from msgl import ops
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    hq, hkv, H, I = CFG8B["num_q_heads"], CFG8B["num_kv_heads"], CFG8B["hidden"], CFG8B["inter"]
    if args.case == "breakdown":
        return run_breakdown(args, dev)
    if args.case == "extend":  # the 32B chunked prefill's attention at a TP8 rank: 2048 queries
        # (8 q heads, 1 kv head) over the last chunk of an 8192-token prompt, causal
        CH, PL, hq8, hkv8 = 2048, 8192, 8, 1
        num_pages, ptp = scattered_pages([PL], seed=3)
        kp = ops.fill_normal_(torch.empty(num_pages * PAGE, hkv8 * 128, dtype=torch.bfloat16, device=dev), seed=4)
        vp = ops.fill_normal_(torch.empty_like(kp), seed=4, stream_id=1)
        q = ops.fill_normal_(torch.empty(CH, hq8, 128, dtype=torch.bfloat16, device=dev), seed=5)
        ptd = torch.from_numpy(ptp).to(dev)
        seq = torch.tensor([PL], dtype=torch.int32, device=dev)
        qip = torch.tensor([0, CH], dtype=torch.int32, device=dev)
        run = lambda: ops.paged_attention_extend(q, kp, vp, ptd, seq, qip, CH, hq8, hkv8)
        ms = time_kernel(run, args.steps, torch.cuda.current_stream())
        assert ops.device_error() == (0, 0)
        pairs = sum(PL - CH + i + 1 for i in range(CH))
        tf = 4.0 * 128 * pairs * hq8 / (ms * 1e-3) / 1e12
        print(f"case {args.case}: {args.steps} launches ok, {ms * 1e3:.1f} us per launch, "
              f"{tf:.1f} TFLOP/s", flush=True)
        return 0
    if args.case == "attention_ragged":
        B, hq6, hkv6 = 64, CFG06B["num_q_heads"], CFG06B["num_kv_heads"]
        ctx = np.random.default_rng(2).integers(512, 4097, B).astype(np.int32)
        num_pages, ptr = scattered_pages(ctx, seed=3)
        kp = ops.fill_normal_(torch.empty(num_pages * PAGE, hkv6 * 128, dtype=torch.bfloat16, device=dev), seed=4)
        vp = ops.fill_normal_(torch.empty_like(kp), seed=4, stream_id=1)
        q = ops.fill_normal_(torch.empty(B, hq6, 128, dtype=torch.bfloat16, device=dev), seed=5)
        ptd = torch.from_numpy(ptr).to(dev)
        seq = torch.from_numpy(ctx).to(dev)
        ws = ops.attention_workspace(B, int(ctx.max()), hq6, hkv6, dev)
        run = lambda: ops.paged_attention_decode(q, kp, vp, ptd, seq, int(ctx.max()), hq6, hkv6,
                                                 workspace=ws)
    elif args.case == "moe_gate_up":
        T, E, K, Hm, Im = 256, 128, 8, 2048, 768
        lib = msgl.lib()
        s_ = torch.cuda.current_stream().cuda_stream
        rng = np.random.default_rng(7)
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        idd = torch.from_numpy(ids).to(dev)
        off = torch.empty(E + 1, dtype=torch.int32, device=dev)
        tok = torch.empty(T * K, dtype=torch.int32, device=dev)
        pos = torch.empty(T * K, dtype=torch.int32, device=dev)
        msgl.check(lib.msgl_moe_permute(idd.data_ptr(), T, K, E, off.data_ptr(), tok.data_ptr(),
                                        pos.data_ptr(), s_))
        xs = ops.fill_normal_(torch.empty(T * K, Hm, dtype=torch.bfloat16, device=dev), seed=6)
        w = ops.fill_normal_(torch.empty(E, 2 * Im, Hm, dtype=torch.bfloat16, device=dev), seed=7,
                             std=0.02)
        act = torch.empty(T * K, Im, dtype=torch.bfloat16, device=dev)
        gws = torch.zeros(lib.msgl_grouped_gemm_workspace_size(T * K, E), dtype=torch.uint8, device=dev)
        run = lambda: msgl.check(lib.msgl_grouped_gemm_gate_up_silu(
            xs.data_ptr(), w.data_ptr(), act.data_ptr(), off.data_ptr(), E, Im, Hm, T * K,
            gws.data_ptr(), gws.numel(), torch.cuda.current_stream().cuda_stream))
    elif args.case in ("attention", "attention_cascade"):
        num_pages, pt = build_pages()
        kp = torch.empty(num_pages * PAGE, hkv * 128, dtype=torch.bfloat16, device=dev)
        vp = torch.empty_like(kp)
        ops.fill_normal_(kp, seed=4, stream_id=0)
        ops.fill_normal_(vp, seed=4, stream_id=1)
        q = ops.fill_normal_(torch.empty(BATCH, hq, 128, dtype=torch.bfloat16, device=dev), seed=5)
        ptd = torch.from_numpy(pt).to(dev)
        seq = torch.full((BATCH,), CTX, dtype=torch.int32, device=dev)
        if args.case == "attention":
            ws = ops.attention_workspace(BATCH, CTX, hq, hkv, dev)
            run = lambda: ops.paged_attention_decode(q, kp, vp, ptd, seq, CTX, hq, hkv, workspace=ws)
        else:  # the step's kernel: cascade over the 1024-token shared prefix
            n = ops.lib().msgl_paged_attention_cascade_workspace_size(BATCH, CTX, PREFIX // PAGE,
                                                                      hq, hkv, 128)
            ws = torch.zeros(n, dtype=torch.uint8, device=dev)
            run = lambda: ops.paged_attention_decode_cascade(q, kp, vp, ptd, seq, CTX,
                                                             PREFIX // PAGE, hq, hkv, workspace=ws)
    elif args.case == "gemm":
        x = ops.fill_normal_(torch.empty(BATCH, H, dtype=torch.bfloat16, device=dev), seed=6)
        w = ops.fill_normal_(torch.empty(2 * I, H, dtype=torch.bfloat16, device=dev), seed=7,
                             std=0.02)
        ws = ops.gemm_workspace(BATCH, 2 * I, H, dev)
        run = lambda: ops.gate_up_silu(x, w, workspace=ws)
    elif args.case == "gemm_partials":  # o_proj of one layer at 128 tokens as split-K partials
        x = ops.fill_normal_(torch.empty(BATCH, hq * 128, dtype=torch.bfloat16, device=dev), seed=6)
        w = ops.fill_normal_(torch.empty(H, hq * 128, dtype=torch.bfloat16, device=dev), seed=7,
                             std=0.02)
        S = ops.gemm_partials_splits(BATCH, H, hq * 128)
        pbuf = torch.empty(S, BATCH, H, dtype=torch.float32, device=dev)
        run = lambda: ops.linear_partials(x, w, S, out=pbuf)
    elif args.case == "gemm_prefill":  # gate_up + SwiGLU of one layer at 2048 prefill tokens
        x = ops.fill_normal_(torch.empty(2048, H, dtype=torch.bfloat16, device=dev), seed=6)
        w = ops.fill_normal_(torch.empty(2 * I, H, dtype=torch.bfloat16, device=dev), seed=7,
                             std=0.02)
        ws = ops.gemm_workspace(2048, 2 * I, H, dev)
        run = lambda: ops.gate_up_silu(x, w, workspace=ws)
    else:  # gemm_qkv: the qkv projection, a small-N (stream-K) GEMM
        n = (hq + 2 * hkv) * 128
        x = ops.fill_normal_(torch.empty(BATCH, H, dtype=torch.bfloat16, device=dev), seed=6)
        w = ops.fill_normal_(torch.empty(n, H, dtype=torch.bfloat16, device=dev), seed=7, std=0.02)
        ws = ops.gemm_workspace(BATCH, n, H, dev)
        run = lambda: ops.linear(x, w, workspace=ws)
    for _ in range(args.steps):
        run()
    torch.cuda.synchronize()
    assert ops.device_error() == (0, 0)
    print(f"case {args.case}: {args.steps} launches ok", flush=True)
    return 0


def run_breakdown(args, dev):
    """Each kernel of the decode step timed alone with CUDA events at the bench's shapes (one
    layer; weight copies rotated so every launch streams its weights from HBM, as in the step).
    With --tp-shape N the shapes are those of one rank of N-way tensor parallelism (q heads,
    kv heads, intermediate columns and vocab rows divided by N; kv heads at least 1), without the
    all-reduce. Prints one JSON line: per kernel the mean launch time and achieved GB/s."""
    import torch

    from msgl import ops
    tp = max(1, args.tp_shape)
    H = CFG8B["hidden"]
    hq = CFG8B["num_q_heads"] // tp
    hkv = max(1, CFG8B["num_kv_heads"] // tp)
    I = CFG8B["inter"] // tp
    V = -(-CFG8B["vocab"] // tp)
    res = {}

    def timed(name, fns, nbytes, reps=None):
        # the launches are captured in a CUDA graph, so only device time is measured
        reps = reps or max(args.steps, 10)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for f in fns:
                f()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                fns[i % len(fns)]()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        us = e0.elapsed_time(e1) * 1000 / reps
        res[name] = {"us": round(us, 2), "GB/s": round(nbytes / (us * 1e-6) / 1e9, 1)}

    x = ops.fill_normal_(torch.empty(BATCH, H, dtype=torch.bfloat16, device=dev), seed=1)
    act = ops.fill_normal_(torch.empty(BATCH, I, dtype=torch.bfloat16, device=dev), seed=2)
    attn_in = ops.fill_normal_(torch.empty(BATCH, hq * 128, dtype=torch.bfloat16, device=dev), seed=3)
    for name, (n, k, inp, kind) in {"qkv": ((hq + 2 * hkv) * 128, H, x, "bf16"),
                                    "o_proj": (H, hq * 128, attn_in, "bf16"),
                                    "gate_up_silu": (2 * I, H, x, "silu"),
                                    "down": (H, I, act, "bf16")}.items():
        copies = max(1, -(-400_000_000 // (n * k * 2)))  # > 3x the 126 MB L2 in total
        ws = [ops.fill_normal_(torch.empty(n, k, dtype=torch.bfloat16, device=dev), seed=10 + i,
                               std=0.02) for i in range(copies)]
        gws = ops.gemm_workspace(BATCH, n, k, dev)
        if kind == "silu":
            fns = [lambda w=w: ops.gate_up_silu(inp, w, workspace=gws) for w in ws]
        else:
            fns = [lambda w=w: ops.linear(inp, w, workspace=gws) for w in ws]
        timed(name, fns, n * k * 2)
        del ws
    # the same projections as split-K partials (the decode step's path at tensor parallel size 1)
    for name, (n, k, inp) in {"qkv_partials": ((hq + 2 * hkv) * 128, H, x),
                              "o_proj_partials": (H, hq * 128, attn_in),
                              "down_partials": (H, I, act)}.items():
        copies = max(1, -(-400_000_000 // (n * k * 2)))
        ws = [ops.fill_normal_(torch.empty(n, k, dtype=torch.bfloat16, device=dev), seed=10 + i,
                               std=0.02) for i in range(copies)]
        S = ops.gemm_partials_splits(BATCH, n, k)
        pbuf = torch.empty(S, BATCH, n, dtype=torch.float32, device=dev)
        timed(name, [lambda w=w: ops.linear_partials(inp, w, S, out=pbuf) for w in ws], n * k * 2)
        res[name]["splits"] = S
        del ws
    S = ops.gemm_partials_splits(BATCH, H, H)
    pn = torch.randn(S * BATCH * H, dtype=torch.float32, device=dev)
    rr = torch.zeros(BATCH, H, dtype=torch.float32, device=dev)
    nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    timed("add_partials_rmsnorm", [lambda: ops.add_partials_rmsnorm_(pn, x, rr, nw, 1e-6)],
          BATCH * H * (4 * S + 10))
    nq = (hq + 2 * hkv) * 128
    Sq = ops.gemm_partials_splits(BATCH, nq, H)
    qkv_b = ops.fill_normal_(torch.empty(BATCH, nq, dtype=torch.bfloat16, device=dev), seed=22)
    qkv_p = torch.randn(Sq * BATCH * nq, dtype=torch.float32, device=dev)
    kpool = torch.zeros(BATCH * 16, hkv * 128, dtype=torch.bfloat16, device=dev)
    vpool = torch.zeros_like(kpool)
    pos = torch.arange(BATCH, dtype=torch.int32, device=dev)
    cs = torch.randn(BATCH * 128, dtype=torch.float32, device=dev)
    qnw = torch.ones(128, dtype=torch.bfloat16, device=dev)
    timed("qknorm_rope", [lambda: ops.qknorm_rope_store_kv(qkv_b, kpool, vpool, pos, pos, cs, qnw,
                                                           qnw, hq, hkv, 1e-6)], BATCH * nq * 4)
    timed("qknorm_rope_partials", [lambda: ops.qknorm_rope_store_kv_partials(
        qkv_p, kpool, vpool, pos, pos, cs, qnw, qnw, hq, hkv, 1e-6)], BATCH * nq * (4 * Sq + 2))
    del qkv_p, pn
    wl = ops.fill_normal_(torch.empty(V, H, dtype=torch.bfloat16, device=dev), seed=20, std=0.02)
    lws = ops.gemm_workspace(BATCH, V, H, dev)
    timed("lm_head_argmax", [lambda: ops.lm_head_argmax(x, wl, workspace=lws)], V * H * 2)
    del wl
    num_pages, pt = build_pages()
    kp = torch.empty(num_pages * PAGE, hkv * 128, dtype=torch.bfloat16, device=dev)
    vp = torch.empty_like(kp)
    ops.fill_normal_(kp, seed=4, stream_id=0)
    ops.fill_normal_(vp, seed=4, stream_id=1)
    q = ops.fill_normal_(torch.empty(BATCH, hq, 128, dtype=torch.bfloat16, device=dev), seed=5)
    ptd = torch.from_numpy(pt).to(dev)
    seq = torch.full((BATCH,), CTX, dtype=torch.int32, device=dev)
    aws = ops.attention_workspace(BATCH, CTX, hq, hkv, dev)
    unique = (PREFIX + BATCH * (CTX - PREFIX)) * hkv * 128 * 4
    timed("paged_decode", [lambda: ops.paged_attention_decode(q, kp, vp, ptd, seq, CTX, hq, hkv,
                                                               workspace=aws)], unique)
    cws = torch.zeros(ops.lib().msgl_paged_attention_cascade_workspace_size(BATCH, CTX, PREFIX // PAGE,
                                                                            hq, hkv, 128),
                      dtype=torch.uint8, device=dev)
    timed("paged_decode_cascade", [lambda: ops.paged_attention_decode_cascade(
        q, kp, vp, ptd, seq, CTX, PREFIX // PAGE, hq, hkv, workspace=cws)], unique)
    r = torch.zeros(BATCH, H, dtype=torch.float32, device=dev)
    nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    timed("add_rmsnorm", [lambda: ops.add_rmsnorm_(x, r, nw, 1e-6)], BATCH * H * 12)
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) \
        if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    for v in res.values():
        v["frac_hbm"] = round(v["GB/s"] / peak, 3)
    if tp > 1:
        print(json.dumps({"case": "breakdown", "tp_shape": tp, "kernels": res}), flush=True)
        return 0
    # prefill-sized projections (2048 tokens): tensor-bound, reported against the bf16 peak
    tpeak = peaks.get("bf16_tflops", 1590.0)
    mp = 2048
    xp = ops.fill_normal_(torch.empty(mp, H, dtype=torch.bfloat16, device=dev), seed=30)
    for name, (n, kind) in {"prefill_qkv_m2048": ((hq + 2 * hkv) * 128, "bf16"),
                            "prefill_gate_up_silu_m2048": (2 * I, "silu")}.items():
        w = ops.fill_normal_(torch.empty(n, H, dtype=torch.bfloat16, device=dev), seed=31, std=0.02)
        gws = ops.gemm_workspace(mp, n, H, dev)
        f = (lambda: ops.gate_up_silu(xp, w, workspace=gws)) if kind == "silu" else \
            (lambda: ops.linear(xp, w, workspace=gws))
        timed(name, [f], n * H * 2 + mp * H * 2)
        us = res[name]["us"]
        res[name]["TFLOP/s"] = round(2.0 * mp * n * H / (us * 1e-6) / 1e12, 1)
        res[name]["frac_tensor"] = round(res[name]["TFLOP/s"] / tpeak, 3)
        del w
    print(json.dumps({"case": "breakdown", "kernels": res}), flush=True)
    return 0


# ============================================================================== other workloads
# The model shapes of the other benchmark configurations (random-init weights, synthetic inputs
# of each configuration's shape: no dataset is involved).
CFG06B = dict(num_layers=28, hidden=1024, num_q_heads=16, num_kv_heads=8, head_dim=128, inter=3072,
              vocab=151936, eps=1e-6, rope_base=1e6)
CFG32B = dict(num_layers=64, hidden=5120, num_q_heads=64, num_kv_heads=8, head_dim=128, inter=25600,
              vocab=151936, eps=1e-6, rope_base=1e6)
CFG30BA3B = dict(num_layers=48, hidden=2048, num_q_heads=32, num_kv_heads=4, head_dim=128, inter=0,
                 vocab=151936, eps=1e-6, rope_base=1e6, num_experts=128, top_k=8, moe_inter=768,
                 norm_topk=True)


def load_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {}


def scattered_pages(ctx_lens, seed, extra=16):
    """Page tables for requests of the given context lengths, their pages a random permutation
    of the pool (Fisher-Yates with `seed`). Returns (num_pages, page_table [B, width])."""
    per = [-(-int(c) // PAGE) for c in ctx_lens]
    num_pages = sum(per) + extra
    perm = np.random.default_rng(seed).permutation(num_pages).astype(np.int32)
    pt = np.zeros((len(per), max(per)), np.int32)
    off = 0
    for r, n in enumerate(per):
        pt[r, :n] = perm[off:off + n]
        off += n
    return num_pages, pt


def decode_host(pt, ctx, vocab, seed=1):
    """Host arrays of one decode step at contexts `ctx` (each request's last token)."""
    B = len(ctx)
    ctx = np.asarray(ctx, np.int32)
    pos = (ctx - 1).astype(np.int32)
    slots = (pt[np.arange(B), pos // PAGE] * PAGE + pos % PAGE).astype(np.int32)
    return dict(input_ids=np.random.default_rng(seed).integers(0, vocab, B).astype(np.int32),
                positions=pos, slot_mapping=slots, page_table=np.ascontiguousarray(pt),
                seq_lens=ctx.copy(), q_indptr=np.arange(B + 1, dtype=np.int32),
                last_idx=np.arange(B, dtype=np.int32))


def fill_kv(model, layers, hkv_l, dev):
    """Synthetic KV cache contents: every pool N(0, 1) bf16 (seed 4)."""
    import torch

    from msgl import ops
    from msgl.model import device_view
    for l in range(layers):
        k, v, n = model.kv_pool(l)
        for j, ptr in enumerate((k, v)):
            ops.fill_normal_(device_view(ptr, (n * hkv_l * 128,), torch.bfloat16), seed=4,
                             stream_id=2 * l + j, std=1.0)


def time_kernel(fn, reps, stream):
    """Mean device time (ms) of `fn` over `reps` launches on `stream` (CUDA events, after one
    warm-up launch)."""
    import torch
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


class Rig:
    """Per-process setup shared by the workloads: device, stream, rank helpers."""

    def __init__(self, args, rank, world, local_rank):
        import torch
        import torch.distributed as dist

        import msgl
        self.args, self.rank, self.world = args, rank, world
        torch.cuda.set_device(local_rank)
        self.dev = torch.device("cuda", local_rank)
        self.local_rank = local_rank
        self.lib = msgl.lib()
        self.stream = torch.cuda.Stream()
        torch.cuda.set_stream(self.stream)
        self.sp = self.stream.cuda_stream
        self.dist = dist
        self.comm = None
        if world > 1:
            from msgl.model import TPComm
            uid = [TPComm.new_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            self.comm = TPComm(rank, world, uid[0])

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, x):
        if self.world == 1:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def blocks(self, fn):
        return timed_blocks(fn, self.args, self.world, self.dev, self.stream, self.barrier,
                            self.max_over_ranks)

    def model(self, cfg, max_tokens, max_reqs):
        from msgl.model import Qwen3Model
        m = Qwen3Model(cfg, max_tokens=max_tokens, max_reqs=max_reqs, tp_rank=self.rank,
                       tp_size=self.world)
        if self.comm is not None:
            m.set_tp(self.comm)
        m.random_init(seed=0, std=0.02)
        return m

    def launches(self, fn):
        """Kernels of ours launched by one eager call of fn."""
        import torch
        n0 = self.lib.msgl_kernel_launches()
        fn()
        n = self.lib.msgl_kernel_launches() - n0
        torch.cuda.synchronize()
        return int(n)

    def close(self):
        if self.comm is not None:
            self.comm.close()


def contract_line(rig, metric, value, unit, ms, blocks, config, dtype="bf16", **extra):
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": rig.world,
            "steps": rig.args.steps, "warmup": rig.args.warmup, "ms_per_step": ms,
            "blocks_ms_per_step": [round(b, 4) for b in blocks], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (random-init weights, N(0,1) KV, random token ids)",
            "config": config}
    line.update(extra)
    return line


def e2e_host_batch(host, is_decode, max_seq_len, max_q_len, shared=None, tail=None):
    """Pinned host copies of a step's arrays and the msgl_batch (host pointers) for
    msgl_model_step_host."""
    import ctypes as C

    import torch

    from msgl.model import DECODE_TAIL_DETECT, SHARED_PREFIX_DETECT, BatchT
    pinned = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in host.items()}
    B = host["seq_lens"].size
    hb = BatchT(int(host["input_ids"].size), B, int(is_decode), host["page_table"].shape[1],
                max_seq_len, max_q_len,
                *[pinned[k].data_ptr() for k in ("input_ids", "positions", "slot_mapping",
                                                  "page_table", "seq_lens", "q_indptr", "last_idx")],
                SHARED_PREFIX_DETECT if shared is None else shared,
                DECODE_TAIL_DETECT if tail is None else tail)
    out = torch.empty(B, dtype=torch.int32).pin_memory()
    return pinned, hb, out, C.addressof(hb)


# ---------------------------------------------------------------- C2: 0.6B ragged decode
def run_c2(rig):
    """Qwen3-0.6B decode step at batch 64, contexts U[512, 4096] (seed 2), every request's pages a
    random permutation of the pool (seed 3), KV N(0, 1). value: 64 tokens / step (graph replay);
    roofline: the plain paged decode kernel (no shared prefix here) over the 28 layers' pools,
    KV bytes = sum(ctx) x Hkv x 128 x 2 B x 2 per launch."""
    import torch

    import msgl
    from msgl import ops
    from msgl.model import make_step, shard_plan
    B = 64
    cfg = dict(CFG06B, max_position=4096 + PAGE)
    ctx = np.random.default_rng(2).integers(512, 4097, B).astype(np.int32)
    num_pages, pt = scattered_pages(ctx, seed=3)
    plan = shard_plan(cfg["num_q_heads"], cfg["num_kv_heads"], cfg["inter"], cfg["vocab"], rig.rank, rig.world)
    hq, hkv = plan["q_heads"], plan["kv_heads"]
    model = rig.model(cfg, B, B)
    model.alloc_kv(num_pages)
    fill_kv(model, cfg["num_layers"], hkv, rig.dev)
    host = decode_host(pt, ctx, cfg["vocab"])
    sb = make_step(host, True, rig.dev, int(ctx.max()), 1)
    assert sb.struct.shared_prefix_pages == 0
    nxt = torch.empty(B, dtype=torch.int32, device=rig.dev)
    per_step = rig.launches(lambda: model.forward(sb, out=nxt))
    for _ in range(max(rig.args.warmup, 3)):
        model.forward(sb, out=nxt, graph=True)
    with ClockSampler(rig.local_rank) as clk:
        blocks = rig.blocks(lambda: model.forward(sb, out=nxt, graph=True))
    ms = float(np.median(blocks))
    assert ops.device_error() == (0, 0)
    pinned, hb, out_host, hbp = e2e_host_batch(host, True, int(ctx.max()), 1)
    step_host = lambda: msgl.check(rig.lib.msgl_model_step_host(model.h, hbp, out_host.data_ptr(), 1, rig.sp))
    for _ in range(max(rig.args.warmup, 3)):
        step_host()
    blocks_e2e = rig.blocks(step_host)
    assert torch.equal(out_host.to(rig.dev), nxt)
    # roofline: the plain decode kernel alone on every layer's pool
    q = ops.fill_normal_(torch.empty(B, hq, 128, dtype=torch.bfloat16, device=rig.dev), seed=5)
    aout = torch.empty_like(q)
    ws = ops.attention_workspace(B, int(ctx.max()), hq, hkv, rig.dev)
    pt_d, seq_d = sb.tensors["page_table"], sb.tensors["seq_lens"]
    pools = [model.kv_pool(l) for l in range(cfg["num_layers"])]
    li = [0]

    def attn():
        k, v, n = pools[li[0] % len(pools)]
        li[0] += 1
        msgl.check(rig.lib.msgl_paged_attention_decode(
            q.data_ptr(), k, v, n, pt_d.data_ptr(), pt_d.shape[1], seq_d.data_ptr(), B,
            int(ctx.max()), hq, hkv, 128, PAGE, 1.0 / 128 ** 0.5, aout.data_ptr(), ws.data_ptr(),
            ws.numel(), rig.sp))

    attn_ms = time_kernel(attn, 3 * cfg["num_layers"], rig.stream)
    kv_bytes = int(ctx.astype(np.int64).sum()) * hkv * 128 * 2 * 2
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = kv_bytes / (attn_ms * 1e-3) / 1e9
    if rig.rank != 0:
        return 0
    cpu = CpuModelRef(cfg, int(ctx.mean()))
    cpu_val, sample = cpu.sample(B, B, cfg["num_layers"])
    cpu.close()
    line = contract_line(
        rig, "Qwen3-0.6B decode tok/s (batch 64, ctx U[512,4096], permuted pages)", B / (ms * 1e-3),
        UNIT, ms, blocks,
        {"workload": "qwen3-0.6b-decode-ragged", "model_arch": "Qwen3-0.6B", "global_batch": B,
         "seq_len": "U[512,4096] (seed 2), mean %d" % int(ctx.mean()), "page_size": PAGE,
         "pages": "random permutation of the pool (seed 3)", "parallelism": f"tp{rig.world}",
         "l2": "inputs larger than L2 (%.1f GB of KV + 1.2 GB of weights per step)"
               % (kv_bytes * cfg["num_layers"] / 1e9 * rig.world)},
        e2e={"value": B / (float(np.median(blocks_e2e)) * 1e-3), "unit": UNIT,
             "h2d_bytes_per_step": sum(v.nbytes for v in host.values()), "d2h_bytes_per_step": B * 4,
             "ms_per_step": float(np.median(blocks_e2e)),
             "blocks_ms_per_step": [round(b, 4) for b in blocks_e2e]},
        roofline={"kernel": "paged_decode_kernel", "bound": "hbm", "achieved": achieved,
                  "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                  "algorithmic_bytes_per_launch": kv_bytes, "launch_ms": attn_ms,
                  "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        cpu_baseline={"value": cpu_val, "unit": UNIT, "cores": cpu.threads, "kind": "reference",
                      "sample": sample, "extrapolated": True},
        clocks=clk.summary(), gpu_launches=per_step * rig.args.steps,
        gpu_launches_per_step=per_step)
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- C5: 30B-A3B MoE
def run_c5(rig):
    """Qwen3-30B-A3B (48 layers, 128 experts, top-8, moe_intermediate 768): decode step at batch
    256, context 1024 (value, graph replay), and one 4096-token prefill chunk (reported beside
    it). roofline: the grouped expert gate_up + SwiGLU GEMM on a decode step's routing (256
    tokens x top-8 over 128 experts) -- algorithmic bytes = the gate_up weights of the experts
    the routing touches."""
    import torch

    import msgl
    from msgl import ops
    from msgl.model import BatchBuilder, PagePool, Request, make_step, shard_plan
    B, CTXD, PRE = 256, 1024, 4096
    cfg = dict(CFG30BA3B, max_position=PRE + PAGE)
    E, K, H = cfg["num_experts"], cfg["top_k"], cfg["hidden"]
    plan = shard_plan(cfg["num_q_heads"], cfg["num_kv_heads"], cfg["moe_inter"], cfg["vocab"],
                      rig.rank, rig.world)
    hkv = plan["kv_heads"]
    Im = cfg["moe_inter"] // rig.world
    ctx = np.full(B, CTXD, np.int32)
    num_pages, pt = scattered_pages(ctx, seed=3, extra=PRE // PAGE + 16)
    model = rig.model(cfg, PRE, B)
    model.alloc_kv(num_pages)
    fill_kv(model, cfg["num_layers"], hkv, rig.dev)
    host = decode_host(pt, ctx, cfg["vocab"])
    sb = make_step(host, True, rig.dev, CTXD, 1)
    nxt = torch.empty(B, dtype=torch.int32, device=rig.dev)
    per_step = rig.launches(lambda: model.forward(sb, out=nxt))
    for _ in range(max(rig.args.warmup, 3)):
        model.forward(sb, out=nxt, graph=True)
    with ClockSampler(rig.local_rank) as clk:
        blocks = rig.blocks(lambda: model.forward(sb, out=nxt, graph=True))
    ms = float(np.median(blocks))
    pinned, hb, out_host, hbp = e2e_host_batch(host, True, CTXD, 1)
    step_host = lambda: msgl.check(rig.lib.msgl_model_step_host(model.h, hbp, out_host.data_ptr(), 1, rig.sp))
    for _ in range(max(rig.args.warmup, 3)):
        step_host()
    blocks_e2e = rig.blocks(step_host)
    # the 4096-token prefill chunk: one request on the pages no decode request holds
    pool = PagePool(0)
    pool.free = sorted(set(range(num_pages)) - set(pt.ravel().tolist()))
    req = Request(list(np.random.default_rng(7).integers(0, cfg["vocab"], PRE)))
    sbp = BatchBuilder(pool).build([req], decode=False, device=rig.dev)
    nxp = torch.empty(1, dtype=torch.int32, device=rig.dev)
    for _ in range(2):
        model.forward(sbp, out=nxp, graph=True)
    blocks_pre = rig.blocks(lambda: model.forward(sbp, out=nxp, graph=True))
    ms_pre = float(np.median(blocks_pre))
    assert ops.device_error() == (0, 0)
    # roofline: grouped gate_up + SwiGLU alone on a decode step's routing
    rng = np.random.default_rng(8)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(B)]).astype(np.int32)
    ids_d = torch.from_numpy(ids).to(rig.dev)
    off = torch.zeros(E + 1, dtype=torch.int32, device=rig.dev)
    tok = torch.empty(B * K, dtype=torch.int32, device=rig.dev)
    pos = torch.empty(B * K, dtype=torch.int32, device=rig.dev)
    msgl.check(rig.lib.msgl_moe_permute(ids_d.data_ptr(), B, K, E, off.data_ptr(), tok.data_ptr(),
                                        pos.data_ptr(), rig.sp))
    xs = ops.fill_normal_(torch.empty(B * K, H, dtype=torch.bfloat16, device=rig.dev), seed=9)
    wgu = ops.fill_normal_(torch.empty(E, 2 * Im, H, dtype=torch.bfloat16, device=rig.dev), seed=10,
                           std=0.02)
    act = torch.empty(B * K, Im, dtype=torch.bfloat16, device=rig.dev)
    gws = torch.zeros(rig.lib.msgl_grouped_gemm_workspace_size(B * K, E), dtype=torch.uint8,
                      device=rig.dev)
    gu = lambda: msgl.check(rig.lib.msgl_grouped_gemm_gate_up_silu(
        xs.data_ptr(), wgu.data_ptr(), act.data_ptr(), off.data_ptr(), E, Im, H, B * K,
        gws.data_ptr(), gws.numel(), rig.sp))
    gu_ms = time_kernel(gu, 20, rig.stream)
    touched = len(np.unique(ids))
    gu_bytes = touched * 2 * Im * H * 2
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
    if rig.rank != 0:
        return 0
    cpu = CpuModelRef(cfg, CTXD)
    cpu_val, sample = cpu.sample(B, B, cfg["num_layers"])
    cpu.close()
    line = contract_line(
        rig, "Qwen3-30B-A3B decode tok/s (batch 256, ctx 1024)", B / (ms * 1e-3), UNIT, ms, blocks,
        {"workload": "qwen3-30b-a3b", "model_arch": "Qwen3-30B-A3B", "global_batch": B,
         "seq_len": CTXD, "page_size": PAGE, "experts": E, "top_k": K,
         "parallelism": f"tp{rig.world}",
         "prefill_chunk": {"tokens": PRE, "ms": ms_pre, "tok_s": PRE / (ms_pre * 1e-3),
                           "blocks_ms": [round(b, 3) for b in blocks_pre]},
         "l2": "inputs larger than L2 (expert weights ~58 GB + KV 25.8 GB per decode step)"},
        e2e={"value": B / (float(np.median(blocks_e2e)) * 1e-3), "unit": UNIT,
             "h2d_bytes_per_step": sum(v.nbytes for v in host.values()), "d2h_bytes_per_step": B * 4,
             "ms_per_step": float(np.median(blocks_e2e)),
             "blocks_ms_per_step": [round(b, 4) for b in blocks_e2e]},
        roofline={"kernel": "gemm_kernel<grouped, SWIGLU> (experts gate_up)", "bound": "hbm",
                  "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                  "traffic": None, "algorithmic_bytes_per_launch": gu_bytes,
                  "experts_touched": touched, "launch_ms": gu_ms,
                  "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        cpu_baseline={"value": cpu_val, "unit": UNIT, "cores": cpu.threads, "kind": "reference",
                      "sample": sample, "extrapolated": True},
        clocks=clk.summary(), gpu_launches=per_step * rig.args.steps,
        gpu_launches_per_step=per_step)
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- C4: 32B mixed chunked prefill
def run_c4(rig):
    """Qwen3-32B mixed chunked prefill: each step = one 2048-token chunk of one of 4 prompts of
    8192 tokens (chunks in order, 16 distinct steps cycled) + 96 decode requests at contexts
    U[1024, 8192] (seed 2): 2144 tokens per step. The decode requests are the batch's tail
    (decode_tail = 96: split-KV decode kernel for them, extend kernel for the chunk). On N GPUs:
    tensor parallel over the N ranks. On 1 GPU the full model does not fit (64 GB of weights +
    ~125 GB of KV), so the run is ONE RANK OF TP8: the shapes of a TP8 shard (8 q heads, 1 kv
    head, 3200 intermediate columns, 18992 vocab rows) as a standalone model, without the 128
    all-reduces per step. roofline: the chunk's gate_up + SwiGLU GEMM (M = 2144) against the
    sustained bf16 peak; the extend attention of the chunk is reported beside it."""
    import torch

    from msgl import ops
    from msgl.model import make_step, shard_plan
    NDEC, CH, NPROMPT, PLEN = 96, 2048, 4, 8192
    if rig.world == 1:
        cfg = dict(CFG32B, num_q_heads=8, num_kv_heads=1, inter=3200, vocab=-(-151936 // 8))
        par = "tp8 rank shard on 1 GPU (no all-reduce)"
    else:
        cfg = dict(CFG32B)
        par = f"tp{rig.world}"
    cfg["max_position"] = PLEN + PAGE
    plan = shard_plan(cfg["num_q_heads"], cfg["num_kv_heads"], cfg["inter"], cfg["vocab"], rig.rank, rig.world)
    hq, hkv, I_l = plan["q_heads"], plan["kv_heads"], plan["inter_cols"]
    H = cfg["hidden"]
    dctx = np.random.default_rng(2).integers(1024, 8193, NDEC).astype(np.int32)
    # prompts first (4 x 512 pages), then the decode requests' pages, all scattered
    lens = [PLEN] * NPROMPT + list(dctx)
    num_pages, pt_all = scattered_pages(lens, seed=3)
    ppt, dpt = pt_all[:NPROMPT], pt_all[NPROMPT:]
    model = rig.model(cfg, CH + NDEC, NDEC + 1)
    model.alloc_kv(num_pages)
    fill_kv(model, cfg["num_layers"], hkv, rig.dev)
    width = pt_all.shape[1]
    rng = np.random.default_rng(1)
    steps = []
    for k in range(NPROMPT * (PLEN // CH)):
        p, c = k // (PLEN // CH), k % (PLEN // CH)
        pos_c = np.arange(c * CH, (c + 1) * CH, dtype=np.int32)
        dpos = dctx - 1
        positions = np.concatenate([pos_c, dpos]).astype(np.int32)
        slots = np.concatenate([ppt[p, pos_c // PAGE] * PAGE + pos_c % PAGE,
                                dpt[np.arange(NDEC), dpos // PAGE] * PAGE + dpos % PAGE]).astype(np.int32)
        host = dict(input_ids=rng.integers(0, cfg["vocab"], CH + NDEC).astype(np.int32),
                    positions=positions, slot_mapping=slots,
                    page_table=np.ascontiguousarray(np.concatenate([ppt[p:p + 1], dpt])[:, :width]),
                    seq_lens=np.concatenate([[(c + 1) * CH], dctx]).astype(np.int32),
                    q_indptr=np.concatenate([[0], CH + np.arange(NDEC + 1)]).astype(np.int32),
                    last_idx=np.concatenate([[CH - 1], CH + np.arange(NDEC)]).astype(np.int32))
        steps.append((host, make_step(host, False, rig.dev, int(max(PLEN, dctx.max())), CH)))
    assert steps[0][1].struct.decode_tail == NDEC
    nxt = torch.empty(NDEC + 1, dtype=torch.int32, device=rig.dev)
    per_step = rig.launches(lambda: model.forward(steps[0][1], out=nxt))
    it = [0]

    def step():
        model.forward(steps[it[0] % len(steps)][1], out=nxt)
        it[0] += 1

    for _ in range(max(rig.args.warmup, 3)):
        step()
    with ClockSampler(rig.local_rank) as clk:
        blocks = rig.blocks(step)
    ms = float(np.median(blocks))
    # e2e: host arrays through msgl_model_step_host (no graph for a prefill step)
    import ctypes as C

    import msgl
    hbs = [e2e_host_batch(h, False, int(max(PLEN, dctx.max())), CH, shared=0) for h, _ in steps]
    ie = [0]

    def step_host():
        _, _, out_h, hbp = hbs[ie[0] % len(hbs)]
        ie[0] += 1
        msgl.check(rig.lib.msgl_model_step_host(model.h, hbp, out_h.data_ptr(), 0, rig.sp))

    for _ in range(max(rig.args.warmup, 3)):
        step_host()
    blocks_e2e = rig.blocks(step_host)
    assert ops.device_error() == (0, 0)
    # roofline: the chunk step's gate_up + SwiGLU at M = 2144 (tensor-bound)
    M = CH + NDEC
    x = ops.fill_normal_(torch.empty(M, H, dtype=torch.bfloat16, device=rig.dev), seed=6)
    w = ops.fill_normal_(torch.empty(2 * I_l, H, dtype=torch.bfloat16, device=rig.dev), seed=7, std=0.02)
    gws = ops.gemm_workspace(M, 2 * I_l, H, rig.dev)
    g_ms = time_kernel(lambda: ops.gate_up_silu(x, w, workspace=gws), 20, rig.stream)
    flops = 2.0 * M * 2 * I_l * H
    peaks = load_peaks()
    tpeak = peaks.get("bf16_tflops_sustained", 1400.0)
    achieved = flops / (g_ms * 1e-3) / 1e12
    # extend attention of the last chunk (2048 queries over 8192 keys, causal) alone
    kp, vp, nsl = model.kv_pool(0)
    q = ops.fill_normal_(torch.empty(CH, hq, 128, dtype=torch.bfloat16, device=rig.dev), seed=8)
    ao = torch.empty_like(q)
    ptc = torch.from_numpy(np.ascontiguousarray(ppt[:1])).to(rig.dev)
    seqc = torch.tensor([PLEN], dtype=torch.int32, device=rig.dev)
    qip = torch.tensor([0, CH], dtype=torch.int32, device=rig.dev)
    ext = lambda: msgl.check(rig.lib.msgl_paged_attention_extend(
        q.data_ptr(), kp, vp, nsl, ptc.data_ptr(), ptc.shape[1], seqc.data_ptr(), qip.data_ptr(), 1,
        CH, hq, hkv, 128, PAGE, 1.0 / 128 ** 0.5, ao.data_ptr(), rig.sp))
    e_ms = time_kernel(ext, 10, rig.stream)
    # causal FLOPs of the chunk: query i sees 6144 + i + 1 keys; QK^T and PV: 4 x 128 per pair
    pairs = sum(PLEN - CH + i + 1 for i in range(CH))
    e_flops = 4.0 * 128 * pairs * hq
    if rig.rank != 0:
        return 0
    cpu = CpuModelRef(CFG32B, int(dctx.mean()))
    cpu_val, sample = cpu.sample(M, NDEC + 1, CFG32B["num_layers"])
    cpu.close()
    line = contract_line(
        rig, "Qwen3-32B mixed chunked-prefill tok/s (2048-token chunk + 96 decodes per step)",
        M / (ms * 1e-3), UNIT, ms, blocks,
        {"workload": "qwen3-32b-mixed", "model_arch": "Qwen3-32B", "tokens_per_step": M,
         "chunk": CH, "prompts": f"{NPROMPT} x {PLEN}", "decodes": NDEC,
         "decode_ctx": "U[1024,8192] (seed 2)", "page_size": PAGE, "parallelism": par,
         "shard": {"q_heads": hq, "kv_heads": hkv, "inter_cols": I_l, "vocab_rows": plan["vocab_rows"]},
         "l2": "inputs larger than L2 (weights %.1f GB per rank per step)" % (model.weight_bytes() / 1e9)},
        e2e={"value": M / (float(np.median(blocks_e2e)) * 1e-3), "unit": UNIT,
             "h2d_bytes_per_step": sum(v.nbytes for v in steps[0][0].values()),
             "d2h_bytes_per_step": (NDEC + 1) * 4, "ms_per_step": float(np.median(blocks_e2e)),
             "blocks_ms_per_step": [round(b, 4) for b in blocks_e2e]},
        roofline={"kernel": "gemm_sk_kernel<SWIGLU> (chunk gate_up, M 2144)", "bound": "tensor",
                  "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s", "frac": achieved / tpeak,
                  "traffic": None, "algorithmic_flops_per_launch": flops, "launch_ms": g_ms,
                  "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained"
                                 if "bf16_tflops_sustained" in peaks else "fallback",
                  "extend_attention": {"kernel": "paged_extend_kernel"
                                       if os.environ.get("MSGL_EXTEND_TC", "1")[:1] == "0"
                                       else "paged_extend_tc_kernel", "launch_ms": e_ms,
                                       "tflops": e_flops / (e_ms * 1e-3) / 1e12,
                                       "frac_of_sustained": e_flops / (e_ms * 1e-3) / 1e12 / tpeak}},
        cpu_baseline={"value": cpu_val, "unit": UNIT, "cores": cpu.threads, "kind": "reference",
                      "sample": sample + " (full 32B model, one process)", "extrapolated": True},
        clocks=clk.summary(), gpu_launches=per_step * rig.args.steps,
        gpu_launches_per_step=per_step)
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- C1: 0.6B greedy run
def run_c1(rig):
    """Qwen3-0.6B, 4 requests x 128 prompt tokens (seed 1), page size 16: one step = the whole
    greedy run, prefill + 31 decode steps (32 new tokens per request); the decode steps go
    through msgl_model_decode_steps (device-advanced metadata, one CUDA graph). value: new tokens
    per second (128 per run). e2e: the same run through msgl_model_step_host, one call per
    step with host arrays. roofline: the fused lm_head + argmax (the largest single launch:
    151936 x 1024 bf16 = 311 MB)."""
    import torch

    import msgl
    from msgl import ops
    from msgl.model import BatchBuilder, PagePool, Request, make_step
    NREQ, PROMPT, NEW, WIDTH = 4, 128, 32, 12
    cfg = dict(CFG06B, max_position=512)
    num_pages = 64
    model = rig.model(cfg, NREQ * PROMPT, NREQ)
    model.alloc_kv(num_pages)
    prompts = np.random.default_rng(1).integers(0, cfg["vocab"], (NREQ, PROMPT)).tolist()
    reqs = [Request(list(p)) for p in prompts]
    pool = PagePool(num_pages)
    bb = BatchBuilder(pool)
    sbp = bb.build(reqs, decode=False, device=rig.dev, max_pages=WIDTH)
    first = torch.empty(NREQ, dtype=torch.int32, device=rig.dev)
    model.forward(sbp, out=first)
    torch.cuda.synchronize()
    for r, t in zip(reqs, first.cpu().numpy().tolist()):
        r.cached_len = r.device_len
        r.input_ids.append(int(t))
    sbd = bb.build(reqs, decode=True, device=rig.dev, max_pages=WIDTH)
    pristine = {k: v.clone() for k, v in sbd.tensors.items()}
    free0 = torch.tensor(pool.free + [0], dtype=torch.int32, device=rig.dev)
    top0 = torch.tensor([len(pool.free)], dtype=torch.int32, device=rig.dev)
    free, top = free0.clone(), top0.clone()
    log = torch.empty(NEW - 1, NREQ, dtype=torch.int32, device=rig.dev)

    import ctypes as C

    def run(graph=True):
        # prefill (writes the prompt KV, emits token 1), then the metadata of the first decode
        # step restored on the device and 31 device-driven decode steps
        model.forward(sbp, out=first, graph=graph)
        for k, v in pristine.items():
            sbd.tensors[k].copy_(v, non_blocking=True)
        free.copy_(free0, non_blocking=True)
        top.copy_(top0, non_blocking=True)
        msgl.check(rig.lib.msgl_model_decode_steps(model.h, C.addressof(sbd.struct), NEW - 1,
                                                   log.data_ptr(), free.data_ptr(), top.data_ptr(),
                                                   int(graph), rig.sp))

    per_run = rig.launches(lambda: run(graph=False))
    for _ in range(max(rig.args.warmup, 3)):
        run()
    with ClockSampler(rig.local_rank) as clk:
        blocks = rig.blocks(run)
    ms = float(np.median(blocks))
    tokens_dev = [first.cpu().numpy().tolist()] + log.cpu().numpy().tolist()
    # e2e: the scheduler-facing call per step with host arrays. The step metadata (positions,
    # slots, page tables; the page allocation of the reference's LIFO pool) is staged once in
    # persistent pinned buffers, one set per step; each step the host writes the previous step's
    # tokens into its input ids and calls msgl_model_step_host (H2D, step, D2H, sync).
    reqs2 = [Request(list(p)) for p in prompts]
    bb2 = BatchBuilder(PagePool(num_pages))
    staged = []
    for st in range(NEW):
        sbh = bb2.build(reqs2, decode=st > 0, device="cpu", max_pages=WIDTH)
        h = {k: v.numpy() for k, v in sbh.tensors.items()}
        staged.append(e2e_host_batch(h, st > 0, int(h["seq_lens"].max()), 1 if st > 0 else PROMPT,
                                     shared=0, tail=0))
        for r, t in zip(reqs2, tokens_dev[st]):  # lengths only: the ids are rewritten per run
            r.cached_len = r.device_len
            r.input_ids.append(int(t))
    h2d_per_run = sum(sum(v.nbytes for v in pin.values()) for pin, _, _, _ in staged)

    def e2e_run():
        toks = []
        for st, (pin, _, out_h, hbp) in enumerate(staged):
            if st > 0:
                pin["input_ids"].copy_(torch.tensor(toks[-1], dtype=torch.int32))
            msgl.check(rig.lib.msgl_model_step_host(model.h, hbp, out_h.data_ptr(), 1, rig.sp))
            toks.append(out_h.numpy().tolist())
        return toks

    for _ in range(2):
        e2e_run()
    tokens_host = None
    blocks_e2e = []
    for _ in range(rig.args.blocks):
        rig.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(rig.args.steps):
            tokens_host = e2e_run()
        torch.cuda.synchronize()
        blocks_e2e.append(rig.max_over_ranks((time.perf_counter() - t0) * 1e3 / rig.args.steps))
    assert tokens_host == tokens_dev, "device-driven run and host-driven run disagree"
    # roofline: lm_head + argmax alone
    x = ops.fill_normal_(torch.empty(NREQ, cfg["hidden"], dtype=torch.bfloat16, device=rig.dev), seed=3)
    wl = ops.fill_normal_(torch.empty(-(-cfg["vocab"] // rig.world), cfg["hidden"], dtype=torch.bfloat16,
                                      device=rig.dev), seed=4, std=0.02)
    lws = ops.gemm_workspace(NREQ, wl.shape[0], cfg["hidden"], rig.dev)
    lm_ms = time_kernel(lambda: ops.lm_head_argmax(x, wl, workspace=lws), 50, rig.stream)
    lm_bytes = wl.numel() * 2
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = lm_bytes / (lm_ms * 1e-3) / 1e9
    assert ops.device_error() == (0, 0)
    if rig.rank != 0:
        return 0
    cpu = CpuModelRef(cfg, PROMPT + NEW // 2)
    _, sample = cpu.sample(1, 1, 1)
    H, V = cfg["hidden"], cfg["vocab"]
    # tokens through the layers per run: the prompts, then one per request per decode step
    tok_layers = NREQ * PROMPT + NREQ * (NEW - 1)
    w_layer, w_lm = cpu._timed_pair()
    run_s = (tok_layers * cfg["num_layers"] * w_layer + NREQ * NEW * w_lm) / cpu.threads
    cpu.close()
    line = contract_line(
        rig, "Qwen3-0.6B greedy generation tok/s (4 x 128-token prompts, 32 new tokens each)",
        NREQ * NEW / (ms * 1e-3), UNIT, ms, blocks,
        {"workload": "qwen3-0.6b-greedy", "model_arch": "Qwen3-0.6B", "requests": NREQ,
         "prompt": PROMPT, "new_tokens": NEW, "page_size": PAGE, "parallelism": f"tp{rig.world}",
         "step": "one whole run: prefill + 31 decode steps",
         "l2": "weights 1.2 GB read per decode step (> L2)"},
        e2e={"value": NREQ * NEW / (float(np.median(blocks_e2e)) * 1e-3), "unit": UNIT,
             "h2d_bytes_per_step": h2d_per_run, "d2h_bytes_per_step": NEW * NREQ * 4,
             "ms_per_step": float(np.median(blocks_e2e)),
             "blocks_ms_per_step": [round(b, 4) for b in blocks_e2e],
             "timing": "host wall clock around 32 msgl_model_step_host calls per run"},
        roofline={"kernel": "gemm_rows_kernel<ARGMAX> (lm_head + greedy)", "bound": "hbm",
                  "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                  "traffic": None, "algorithmic_bytes_per_launch": lm_bytes, "launch_ms": lm_ms,
                  "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        cpu_baseline={"value": NREQ * NEW / run_s, "unit": UNIT, "cores": cpu.threads,
                      "kind": "reference", "extrapolated": True,
                      "sample": f"{cpu.threads} tokens x 1 of 28 layers + {cpu.threads} tokens x "
                                f"lm_head (reference Linear::forward; attention over {PROMPT + NEW // 2} "
                                f"tokens, C restatement), extrapolated to {tok_layers} tokens x 28 "
                                f"layers + {NREQ * NEW} lm_head rows per run; fp32"},
        clocks=clk.summary(), gpu_launches=per_run * rig.args.steps, gpu_launches_per_step=per_run,
        greedy_tokens_device_equal_host=True)
    print(json.dumps(line), flush=True)
    return 0


WORKLOADS = {"qwen3-0.6b-greedy": run_c1, "qwen3-0.6b-decode-ragged": run_c2,
             "qwen3-32b-mixed": run_c4, "qwen3-30b-a3b": run_c5}


def run_workload(args, rank, world, local_rank):
    rig = Rig(args, rank, world, local_rank)
    try:
        return WORKLOADS[args.workload](rig)
    finally:
        import gc
        gc.collect()  # models (and their graphs) go before the communicator
        rig.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tp-shape", type=int, default=1,
                    help="--case breakdown: the shapes of one rank of this tensor-parallel size")
    ap.add_argument("--blocks", type=int, default=3,
                    help="timed blocks of --steps steps each; the median block is reported")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="qwen3-8b-decode",
                    choices=["qwen3-8b-decode", *WORKLOADS],
                    help="qwen3-8b-decode: the headline (default); the others: the remaining "
                         "benchmark configurations")
    ap.add_argument("--case", choices=["attention", "attention_cascade", "gemm", "gemm_qkv",
                                       "gemm_partials", "gemm_prefill", "breakdown", "extend",
                                       "attention_ragged", "moe_gate_up"],
                    default=None,
                    help="run one kernel of the step on a small single-layer case (profiling)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference_arm(args, rank)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        if args.workload != "qwen3-8b-decode":
            return run_workload(args, rank, world, local_rank)
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
