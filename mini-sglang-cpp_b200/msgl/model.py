"""Python handle on the C++ executor (include/msgl_engine.h) and host-side batch building.

``PagePool`` mirrors KVCachePool's free list (src/cache/kvcache.cpp:16-32: pages handed out
LIFO from [0..N-1], so N-1 first); ``BatchBuilder`` turns per-request state into the step
metadata of Scheduler::step (src/scheduler/scheduler.cpp:83-106: prefill positions
cached_len..device_len-1, decode position device_len-1), allocating ceil(len / page_size)
pages per request (the reference allocates one page per token, D12).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import check, lib

P, I, I64, F, U64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64


class ModelConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("num_layers", "hidden", "num_q_heads", "num_kv_heads",
                                        "head_dim", "inter", "vocab", "num_experts", "top_k",
                                        "moe_inter", "norm_topk")] + \
               [("eps", C.c_float), ("rope_base", C.c_float)] + \
               [(n, C.c_int) for n in ("max_position", "max_tokens", "max_reqs", "tp_rank", "tp_size")]


class BatchT(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("num_tokens", "num_reqs", "is_decode", "max_pages",
                                        "max_seq_len", "max_q_len")] + \
               [(n, C.c_void_p) for n in ("input_ids", "positions", "slot_mapping", "page_table",
                                           "seq_lens", "q_indptr", "last_idx")] + \
               [("shared_prefix_pages", C.c_int), ("decode_tail", C.c_int)]


class StopRules(C.Structure):
    _fields_ = [("max_new_tokens", C.c_void_p), ("ignore_eos", C.c_void_p), ("stop_ids", C.c_void_p),
                ("num_stop_ids", C.c_int), ("finished", C.c_void_p), ("generated", C.c_void_p)]


STEP_TOKENS_FROM_PREV = 2  # msgl_model_step_host_async: decode input ids from the previous step
SHARED_PREFIX_DETECT = -1  # msgl_model_step_host computes it from the host page table
DECODE_TAIL_DETECT = -1    # msgl_model_step_host computes it from the host q_indptr


def decode_tail(q_indptr: np.ndarray) -> int:
    """Trailing requests with exactly one query row (a mixed batch's decode requests), fewer
    than the batch."""
    ql = np.diff(np.asarray(q_indptr))
    n = 0
    while n < ql.size - 1 and ql[ql.size - 1 - n] == 1:
        n += 1
    return n


def shared_prefix_pages(page_table: np.ndarray, seq_lens: np.ndarray, page_size: int = 16) -> int:
    """Leading page-table columns holding the same page in every row and covered by every
    context (0 for fewer than two requests): the prefix the cascade decode attends once."""
    B = page_table.shape[0]
    if B < 2:
        return 0
    cap = min(page_table.shape[1], int(np.min(seq_lens)) // page_size)
    same = np.all(page_table[:, :cap] == page_table[0:1, :cap], axis=0)
    return int(cap if same.all() else np.argmin(same))


def _engine():
    return lib()


def _s():
    return torch.cuda.current_stream().cuda_stream


class _CudaArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3}


def device_view(ptr: int, shape, dtype) -> torch.Tensor:
    """A torch view (no copy) of executor-owned device memory."""
    if dtype == torch.bfloat16:
        return torch.as_tensor(_CudaArray(ptr, shape, "<i2"), device="cuda").view(torch.bfloat16)
    ts = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, ts), device="cuda")


# ---------------------------------------------------------------------------- host metadata
class PagePool:
    """KVCachePool free list (kvcache.cpp:16-32): LIFO from [0..N-1]."""

    def __init__(self, num_pages: int):
        self.free = list(range(num_pages))

    def allocate(self) -> int:
        if not self.free:
            raise RuntimeError("KV Cache OOM: No free pages available")
        return self.free.pop()

    def release(self, page: int) -> None:
        self.free.append(page)

    def num_free(self) -> int:
        return len(self.free)


class RadixCache:
    """msgl_radix_*: the page-granular prefix cache (host side)."""

    def __init__(self, page_size: int = 16):
        self.L = lib()
        self.P = page_size
        h = C.c_void_p()
        check(self.L.msgl_radix_create(page_size, C.byref(h)))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self.L.msgl_radix_destroy(self.h)
            self.h = None

    def match(self, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(max(1, len(t) // self.P), np.int32)
        m, node = C.c_int(0), C.c_int64(0)
        check(self.L.msgl_radix_match(self.h, t.ctypes.data, len(t), out.ctypes.data, out.size,
                                      C.byref(m), C.byref(node)))
        return m.value, out[: m.value // self.P].tolist(), node.value

    def insert(self, tokens, pages):
        """Returns (tokens already cached, the caller's pages to free, node)."""
        t = np.ascontiguousarray(tokens, np.int32)
        pg = np.ascontiguousarray(pages, np.int32)
        if pg.size < len(t) // self.P:
            raise ValueError("insert: fewer pages than full pages of tokens")
        dup = np.zeros(max(1, pg.size), np.int32)
        present, nd, node = C.c_int(0), C.c_int(0), C.c_int64(0)
        check(self.L.msgl_radix_insert(self.h, t.ctypes.data, len(t), pg.ctypes.data,
                                       C.byref(present), dup.ctypes.data, C.byref(nd), C.byref(node)))
        return present.value, dup[: nd.value].tolist(), node.value

    def lock(self, node: int, delta: int = 1):
        check(self.L.msgl_radix_lock(self.h, node, delta))

    def evict(self, num_pages: int):
        out = np.zeros(max(1, num_pages), np.int32)
        n = C.c_int(0)
        check(self.L.msgl_radix_evict(self.h, num_pages, out.ctypes.data, C.byref(n)))
        return out[: n.value].tolist()

    def size(self):
        a, b = C.c_int(0), C.c_int(0)
        check(self.L.msgl_radix_size(self.h, C.byref(a), C.byref(b)))
        return a.value, b.value


@dataclass
class Request:
    """The Req fields the step needs (include/minisgl/core/types.h:29-60)."""
    input_ids: list
    cached_len: int = 0
    pages: list = field(default_factory=list)

    @property
    def device_len(self) -> int:
        return len(self.input_ids)


@dataclass
class StepBatch:
    """Device tensors of one step plus the msgl_batch struct pointing at them."""
    tensors: dict
    struct: BatchT
    num_reqs: int


class BatchBuilder:
    def __init__(self, pool: PagePool, page_size: int = 16):
        self.pool, self.P = pool, page_size

    def _ensure_pages(self, req: Request, upto_len: int):
        need = (upto_len + self.P - 1) // self.P
        while len(req.pages) < need:
            req.pages.append(self.pool.allocate())

    def build(self, reqs: list, decode: bool, device="cuda", max_pages: int | None = None) -> StepBatch:
        ids, pos, slots, seq, qlens = [], [], [], [], []
        for r in reqs:
            if decode:  # scheduler.cpp:93-95
                toks = [(r.input_ids[-1], r.device_len - 1)]
            else:       # scheduler.cpp:88-92
                toks = [(r.input_ids[i], i) for i in range(r.cached_len, r.device_len)]
            self._ensure_pages(r, r.device_len)
            for t, p in toks:
                ids.append(t)
                pos.append(p)
                slots.append(r.pages[p // self.P] * self.P + p % self.P)
            seq.append(r.device_len)
            qlens.append(len(toks))
        width = max_pages or max(len(r.pages) for r in reqs)
        pt = np.zeros((len(reqs), width), np.int32)
        for i, r in enumerate(reqs):
            pt[i, : len(r.pages)] = r.pages
        indptr = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
        host = dict(input_ids=np.array(ids, np.int32), positions=np.array(pos, np.int32),
                    slot_mapping=np.array(slots, np.int32), page_table=pt,
                    seq_lens=np.array(seq, np.int32), q_indptr=indptr,
                    last_idx=(indptr[1:] - 1).astype(np.int32))
        return make_step(host, decode, device, max(seq), max(qlens))


def make_step(host: dict, decode: bool, device, max_seq_len: int, max_q_len: int) -> StepBatch:
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in host.items()}
    B = t["seq_lens"].numel()
    sp = shared_prefix_pages(np.asarray(host["page_table"]), np.asarray(host["seq_lens"])) if decode else 0
    tail = 0 if decode else decode_tail(host["q_indptr"])
    st = BatchT(t["input_ids"].numel(), B, int(decode), t["page_table"].shape[1], max_seq_len,
                max_q_len, *[t[k].data_ptr() for k in ("input_ids", "positions", "slot_mapping",
                                                        "page_table", "seq_lens", "q_indptr",
                                                        "last_idx")], sp, tail)
    return StepBatch(t, st, B)


# ---------------------------------------------------------------------------- executor
def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).reshape(a.shape)


class Qwen3Model:
    def __init__(self, cfg: dict, max_tokens: int, max_reqs: int, tp_rank: int = 0,
                 tp_size: int = 1):
        self.L = _engine()
        self.cfg = cfg
        c = ModelConfig(cfg["num_layers"], cfg["hidden"], cfg["num_q_heads"], cfg["num_kv_heads"],
                        cfg.get("head_dim", 128), cfg.get("inter", 0), cfg["vocab"],
                        cfg.get("num_experts", 0), cfg.get("top_k", 0), cfg.get("moe_inter", 0),
                        int(cfg.get("norm_topk", True)), cfg.get("eps", 1e-6),
                        cfg.get("rope_base", 1e6), cfg["max_position"], max_tokens, max_reqs,
                        tp_rank, tp_size)
        h = C.c_void_p()
        check(self.L.msgl_model_create(C.addressof(c), C.addressof(h)))
        self.h = h

    def __del__(self):
        h = getattr(self, "h", None)
        if h is not None and h.value:
            self.L.msgl_model_destroy(h)
            self.h = None

    def random_init(self, seed: int = 0, std: float = 0.02):
        check(self.L.msgl_model_random_init(self.h, seed, std, _s()))

    def set_weight(self, name: str, arr: np.ndarray):
        bits = to_bf16_bits(arr)
        check(self.L.msgl_model_set_weight(self.h, name.encode(), bits.ctypes.data, bits.size, _s()))

    def set_weight_bits(self, name: str, bits: np.ndarray):
        """The same from bf16 bit patterns (uint16) of the full tensor."""
        bits = np.ascontiguousarray(bits, dtype=np.uint16)
        check(self.L.msgl_model_set_weight(self.h, name.encode(), bits.ctypes.data, bits.size, _s()))

    def set_weights(self, named: dict):
        for k, v in named.items():
            self.set_weight(k, v)

    def weight_bytes(self) -> int:
        return self.L.msgl_model_weight_bytes(self.h)

    def load_safetensors(self, model_dir: str):
        """Weights from a Hugging Face safetensors checkpoint directory (msgl_model_load_safetensors)."""
        check(self.L.msgl_model_load_safetensors(self.h, os.fsencode(model_dir), _s()))

    def alloc_kv(self, num_pages: int, page_size: int = 16):
        check(self.L.msgl_model_alloc_kv(self.h, num_pages, page_size, _s()))

    def kv_pool(self, layer: int):
        k, v, n = C.c_void_p(), C.c_void_p(), C.c_int64()
        check(self.L.msgl_model_kv_pool(self.h, layer, C.addressof(k), C.addressof(v), C.addressof(n)))
        return k.value, v.value, n.value

    def forward(self, step: StepBatch, logits: bool = False, out=None, graph: bool = False):
        B = step.num_reqs
        dev = step.tensors["input_ids"].device
        nxt = out if out is not None else torch.empty(B, dtype=torch.int32, device=dev)
        lg = torch.empty(B, self.cfg["vocab"], dtype=torch.float32, device=dev) if logits else None
        check(self.L.msgl_model_forward(self.h, C.addressof(step.struct), nxt.data_ptr(),
                                        None if lg is None else lg.data_ptr(), int(graph), _s()))
        return (nxt, lg) if logits else nxt

    def decode_steps(self, step: StepBatch, num_steps: int, free_pages, free_top, graph: bool = True):
        """msgl_model_decode_steps: num_steps greedy decode steps on the device from `step` (its
        arrays are advanced in place); returns the ids, [num_steps, B] int32 on the device."""
        B = step.num_reqs
        log = torch.empty(num_steps, B, dtype=torch.int32, device=step.tensors["input_ids"].device)
        check(self.L.msgl_model_decode_steps(self.h, C.addressof(step.struct), num_steps,
                                             log.data_ptr(), free_pages.data_ptr(),
                                             free_top.data_ptr(), int(graph), _s()))
        return log

    def decode_steps_stop(self, step: StepBatch, num_steps: int, free_pages, free_top,
                          max_new_tokens, stop_ids, ignore_eos=None, finished=None,
                          generated=None, graph: bool = True):
        """msgl_model_decode_steps_stop: decode steps with the finish rules applied on the device.
        Returns (token log [num_steps, B] with -1 after a request finished, finished, generated)."""
        dev = step.tensors["input_ids"].device
        B = step.num_reqs
        i32 = lambda a: torch.as_tensor(np.asarray(a, np.int32), device=dev)
        mx, sid = i32(max_new_tokens), i32(stop_ids)
        ign = i32(ignore_eos) if ignore_eos is not None else None
        fin = finished if finished is not None else torch.zeros(B, dtype=torch.int32, device=dev)
        gen = generated if generated is not None else torch.zeros(B, dtype=torch.int32, device=dev)
        rules = StopRules(mx.data_ptr(), None if ign is None else ign.data_ptr(), sid.data_ptr(),
                          sid.numel(), fin.data_ptr(), gen.data_ptr())
        log = torch.empty(num_steps, B, dtype=torch.int32, device=dev)
        check(self.L.msgl_model_decode_steps_stop(self.h, C.addressof(step.struct), num_steps,
                                                  log.data_ptr(), free_pages.data_ptr(),
                                                  free_top.data_ptr(), C.addressof(rules),
                                                  int(graph), _s()))
        torch.cuda.current_stream().synchronize()  # the rule arrays above are local
        return log, fin, gen

    def set_tp(self, comm):
        self.tp = comm
        check(self.L.msgl_model_set_tp(self.h, comm.h if comm is not None else None))

    def set_num_layers_run(self, n: int):
        check(self.L.msgl_model_set_num_layers_run(self.h, n))

    def hidden(self, T: int):
        x, r = C.c_void_p(), C.c_void_p()
        check(self.L.msgl_model_debug_hidden(self.h, C.addressof(x), C.addressof(r)))
        return x.value, r.value


# ---------------------------------------------------------------------------- tensor parallel
class TPComm:
    """msgl_tp (NCCL) of this rank. `unique_id` comes from rank 0's `TPComm.new_unique_id()` and
    reaches the other ranks through the launcher (torch.distributed broadcast in the bench)."""

    def __init__(self, rank: int, world: int, unique_id: bytes):
        self.L = lib()
        buf = C.create_string_buffer(unique_id, len(unique_id))
        h = C.c_void_p()
        check(self.L.msgl_tp_init(rank, world, buf, C.addressof(h)))
        self.h, self.rank, self.world = h, rank, world

    @staticmethod
    def new_unique_id() -> bytes:
        L = lib()
        n = L.msgl_tp_unique_id_size()
        buf = C.create_string_buffer(n)
        check(L.msgl_tp_get_unique_id(buf))
        return buf.raw

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.L.msgl_tp_destroy(self.h)
            self.h = None


def shard_plan(num_q_heads, num_kv_heads, inter, vocab, rank, world):
    """msgl_tp_shard_plan as a dict (host only)."""
    out = (C.c_int * 8)()
    check(lib().msgl_tp_shard_plan(num_q_heads, num_kv_heads, inter, vocab, rank, world, out))
    keys = ("q_head0", "q_heads", "kv_head0", "kv_heads", "inter0", "inter_cols", "vocab0", "vocab_rows")
    return dict(zip(keys, list(out)))
