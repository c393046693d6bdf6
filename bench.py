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
class CpuReference:
    """The decode step on the reference CPU code, timed on a bounded sample.

    Each worker thread carries one token through one layer's four projections (the reference's
    Linear::forward, weights held in persistent Linear objects as in a loaded model) and one
    request's attention over the 2048-token context (the C restatement: the reference has no
    paged / GQA attention), then one token through lm_head. `threads` tokens therefore advance
    one layer per sample; the full step (128 tokens x 36 layers + lm_head) extrapolates
    linearly."""

    def __init__(self, threads=None):
        from oracle import Oracle, RefLib
        self.ref, self.orc = RefLib(), Oracle()
        t = threads or min(CPU_THREADS, os.cpu_count() or 1)
        self.threads = max(1, t)
        H, I, V, D = CFG8B["hidden"], CFG8B["inter"], CFG8B["vocab"], 128
        hq, hkv = CFG8B["num_q_heads"], CFG8B["num_kv_heads"]
        self.dims = (H, V, D, hq, hkv)
        L = self.ref.lib
        self.handles = []
        for n, k in [((hq + 2 * hkv) * D, H), (H, hq * D), (2 * I, H), (H, I)]:
            w = np.full((n, k), 0.01, np.float32)  # values do not change fp32 loop timing
            self.handles.append((L.ref_linear_create(w.ctypes.data, k, n), n, k))
        wl = np.full((V, H), 0.01, np.float32)
        self.lm = L.ref_linear_create(wl.ctypes.data, H, V)
        ctx_pages = CTX // PAGE
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

    def sample(self, layers=36):
        H, V, D, hq, hkv = self.dims
        L = self.ref.lib

        def layer_worker():
            for h, n, k in self.handles:
                xin = np.full((1, k), 0.1, np.float32)
                out = np.empty((1, n), np.float32)
                L.ref_linear_run(h, xin.ctypes.data, 1, out.ctypes.data)
            q = np.full((1, hq * D), 0.01, np.float32)
            self.orc.paged_attention(q, self.kp, self.vp, self.pt, [CTX], [0, 1], hq, hkv, D, PAGE)

        def lm_worker():
            xin = np.full((1, H), 0.1, np.float32)
            out = np.empty((1, V), np.float32)
            L.ref_linear_run(self.lm, xin.ctypes.data, 1, out.ctypes.data)

        w_layer = self._timed(layer_worker)
        w_lm = self._timed(lm_worker)
        step_s = BATCH / self.threads * (layers * w_layer + w_lm)
        desc = (f"{self.threads} tokens x 1 of 36 layers (4 projections, reference "
                f"Linear::forward; attention over 2048 tokens, C restatement) + {self.threads} "
                f"tokens x lm_head, extrapolated to 128 tokens x 36 layers; fp32")
        return BATCH / step_s, desc


def run_reference_arm(args, rank):
    if rank != 0:
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

    # ---- roofline: the step's decode attention (cascade over the shared prefix) alone, every
    # layer's pool
    hq, hkv = hq_l, hkv_l  # this rank's heads
    q = torch.empty(BATCH, hq, 128, dtype=torch.bfloat16, device=dev)
    ops.fill_normal_(q, seed=5, std=1.0)
    aout = torch.empty_like(q)
    shared = int(sb.struct.shared_prefix_pages)
    assert shared == PREFIX // PAGE, shared
    wsn = lib.msgl_paged_attention_cascade_workspace_size(BATCH, CTX, shared, hq, hkv, 128)
    ws = torch.zeros(wsn, dtype=torch.uint8, device=dev)
    pt_d, seq_d = sb.tensors["page_table"], sb.tensors["seq_lens"]

    def attn(l):
        k, v, n = pools[l]
        msgl.check(lib.msgl_paged_attention_decode_cascade(
            q.data_ptr(), k, v, n, pt_d.data_ptr(), pt_d.shape[1], seq_d.data_ptr(), BATCH, CTX,
            shared, hq, hkv, 128, PAGE, 1.0 / 128 ** 0.5, aout.data_ptr(), ws.data_ptr(),
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
            "roofline": {"kernel": "paged_decode_cascade_kernel", "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         # the capture is of 8 kv heads; a TP rank reads its own heads only
                         "traffic": PAGED_DECODE_TRAFFIC_BYTES * hkv // CFG8B["num_kv_heads"],
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
    split-K partials; `gemm_prefill`: gate_up + SwiGLU at 2048 tokens."""
    import torch

    import msgl
    from msgl import ops
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    hq, hkv, H, I = CFG8B["num_q_heads"], CFG8B["num_kv_heads"], CFG8B["hidden"], CFG8B["inter"]
    if args.case == "breakdown":
        return run_breakdown(args, dev)
    if args.case in ("attention", "attention_cascade"):
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
    ap.add_argument("--case", choices=["attention", "attention_cascade", "gemm", "gemm_qkv",
                                       "gemm_partials", "gemm_prefill", "breakdown"], default=None,
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
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
