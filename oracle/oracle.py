"""numpy wrappers over the checker libraries (test infrastructure only).

* ``Oracle``  -- oracle/liboracle.so, the C restatement of the reference path (msgl_oracle.c).
* ``RefLib``  -- oracle/_ref/libref_harness.so, the reference's own compiled CPU sources.

Only tests, ``__graft_entry__.smoke`` and bench.py's CPU-baseline leg import this module, and
only as the checker / the timed CPU reference. The product library never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_harness.so")
# The reference source tree (read-only, only needed to build _ref): MSGL_REFERENCE_SRC.
REFERENCE_SRC = os.environ.get("MSGL_REFERENCE_SRC", "")

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
I64, I32, F32, VP = C.c_int64, C.c_int, C.c_float, C.c_void_p


def json_include_dir() -> str:
    """The nlohmann_json v3.11.3 headers vendored in this interpreter's site-packages."""
    import sysconfig
    return os.path.join(sysconfig.get_paths()["purelib"], "include", "cudnn_frontend", "thirdparty")


def build(with_ref: bool | None = None, reference_src: str | None = None) -> None:
    """Compile liboracle.so, and _ref when the reference sources are given (argument or
    MSGL_REFERENCE_SRC) and present."""
    src = reference_src if reference_src is not None else REFERENCE_SRC
    targets, extra = ["oracle"], []
    if with_ref is None:
        with_ref = bool(src) and os.path.isdir(src)
    if with_ref:
        targets.append("ref")
        extra = [f"REF={src}", f"JSON_INC={json_include_dir()}"]
    subprocess.run(["make", "-s", "-C", HERE, *extra, *targets], check=True)


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even) and widen back to fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(a.shape)


def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).reshape(a.shape)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class Oracle:
    """The C restatement. Every method mirrors one function of msgl_oracle.h."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(with_ref=False)
        L = self.lib = C.CDLL(path)
        L.oracle_embedding.argtypes = [f32p, I64, I64, i32p, I64, f32p]
        L.oracle_rmsnorm.argtypes = [f32p, f32p, I64, I64, F32, f32p]
        L.oracle_add_rmsnorm.argtypes = [f32p, f32p, f32p, I64, I64, F32, I32]
        L.oracle_linear.argtypes = [f32p, f32p, VP, I64, I64, I64, f32p]
        L.oracle_swiglu.argtypes = [f32p, f32p, I64, f32p]
        L.oracle_rope_table.argtypes = [I32, I32, F32, f32p]
        L.oracle_rope.argtypes = [f32p, i32p, I64, I32, I32, f32p]
        L.oracle_store_kv_page.argtypes = [f32p, f32p, f32p, f32p, i32p, I32, I32, I32, I64]
        L.oracle_store_kv_slots.argtypes = [f32p, f32p, f32p, f32p, i32p, I64, I64]
        L.oracle_paged_attention.argtypes = [f32p, f32p, f32p, i32p, I32, i32p, i32p, I32, I32,
                                             I32, I32, I32, F32, f32p]
        L.oracle_router_topk.argtypes = [f32p, I64, I32, I32, I32, i32p, f32p]
        L.oracle_moe_experts.argtypes = [f32p, i32p, f32p, I64, I32, I32, I32, VP, VP, f32p]
        L.oracle_argmax.argtypes = [f32p, I64, I64, i32p]

    def embedding(self, w, ids):
        w, ids = _f(w), _i(ids)
        out = np.empty((ids.size, w.shape[1]), np.float32)
        self.lib.oracle_embedding(w, w.shape[0], w.shape[1], ids, ids.size, out)
        return out

    def rmsnorm(self, x, w, eps):
        x, w = _f(x), _f(w)
        out = np.empty_like(x)
        H = w.size
        self.lib.oracle_rmsnorm(x, w, x.size // H, H, eps, out)
        return out

    def add_rmsnorm(self, x, residual, w, eps, first=False):
        """Returns (x_out, residual_out); inputs are not modified."""
        x = _f(x).copy()
        r = np.empty_like(x) if first else _f(residual).copy()
        H = w.size
        self.lib.oracle_add_rmsnorm(x, r, _f(w), x.size // H, H, eps, int(first))
        return x, r

    def linear(self, x, w):
        x, w = _f(x), _f(w)
        N, K = w.shape
        T = x.size // K
        out = np.empty((T, N), np.float32)
        self.lib.oracle_linear(x, w, None, T, K, N, out)
        return out

    def swiglu(self, g, u):
        g, u = _f(g), _f(u)
        out = np.empty_like(g)
        self.lib.oracle_swiglu(g, u, g.size, out)
        return out

    def rope_table(self, head_dim, max_pos, base):
        t = np.empty((max_pos, head_dim), np.float32)
        self.lib.oracle_rope_table(head_dim, max_pos, base, t)
        return t

    def rope(self, x, positions, num_heads, head_dim, table):
        x = _f(x).copy()
        pos = _i(positions)
        self.lib.oracle_rope(x, pos, pos.size, num_heads, head_dim, _f(table))
        return x

    def store_kv_page(self, k, v, k_pool, v_pool, page_table, page_size, num_heads, head_dim):
        k, v = _f(k), _f(v)
        T = k.size // (num_heads * head_dim)
        self.lib.oracle_store_kv_page(k, v, k_pool, v_pool, _i(page_table), page_size, num_heads,
                                      head_dim, T)

    def store_kv_slots(self, k, v, k_pool, v_pool, slots):
        k, v, slots = _f(k), _f(v), _i(slots)
        self.lib.oracle_store_kv_slots(k, v, k_pool, v_pool, slots, slots.size, k.size // slots.size)

    def paged_attention(self, q, k_pool, v_pool, page_table, seq_lens, q_indptr, num_q_heads,
                        num_kv_heads, head_dim, page_size, scale=None):
        q = _f(q)
        pt = _i(page_table)
        seq_lens, q_indptr = _i(seq_lens), _i(q_indptr)
        out = np.zeros_like(q)
        if scale is None:
            scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
        self.lib.oracle_paged_attention(q, _f(k_pool), _f(v_pool), pt, pt.shape[1], seq_lens,
                                        q_indptr, seq_lens.size, num_q_heads, num_kv_heads,
                                        head_dim, page_size, scale, out)
        return out

    def router_topk(self, logits, top_k, norm_topk=True):
        logits = _f(logits)
        T, E = logits.shape
        ids = np.empty((T, top_k), np.int32)
        w = np.empty((T, top_k), np.float32)
        self.lib.oracle_router_topk(logits, T, E, top_k, int(norm_topk), ids, w)
        return ids, w

    def moe_experts(self, x, ids, weights, gate_up_ws, down_ws):
        x = _f(x)
        ids, weights = _i(ids), _f(weights)
        T, H = x.shape
        top_k = ids.shape[1]
        inter = down_ws[0].shape[1]
        gu = [_f(w) for w in gate_up_ws]
        dn = [_f(w) for w in down_ws]
        gu_ptrs = (C.c_void_p * len(gu))(*[a.ctypes.data for a in gu])
        dn_ptrs = (C.c_void_p * len(dn))(*[a.ctypes.data for a in dn])
        out = np.empty_like(x)
        self.lib.oracle_moe_experts(x, ids, weights, T, top_k, H, inter,
                                    C.cast(gu_ptrs, C.c_void_p), C.cast(dn_ptrs, C.c_void_p), out)
        return out

    def argmax(self, logits):
        logits = _f(logits)
        out = np.empty(logits.shape[0], np.int32)
        self.lib.oracle_argmax(logits, logits.shape[0], logits.shape[1], out)
        return out


class RefLib:
    """The reference's own CPU code (oracle/_ref), via the shims of ref_harness.cpp."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle ref`")
        L = self.lib = C.CDLL(path)
        L.ref_embedding.argtypes = [f32p, I32, I32, i32p, I32, f32p]
        L.ref_rmsnorm.argtypes = [f32p, f32p, I32, I32, F32, f32p]
        L.ref_add_rmsnorm.argtypes = [f32p, f32p, f32p, I32, I32, F32, I32]
        L.ref_linear.argtypes = [VP, VP, I32, I32, I32, VP]
        L.ref_swiglu.argtypes = [f32p, f32p, I32, f32p]
        L.ref_rope_table.argtypes = [I32, I32, F32, f32p]
        L.ref_rope.argtypes = [f32p, i32p, I32, I32, I32, I32, F32]
        L.ref_attention_mha.argtypes = [f32p, f32p, f32p, I32, I32, I32, f32p]
        L.ref_router.argtypes = [f32p, f32p, I32, I32, I32, I32, I32, i32p, f32p]
        L.ref_pool_create.argtypes = [I32, I32]
        L.ref_pool_create.restype = VP
        L.ref_pool_destroy.argtypes = [VP]
        L.ref_pool_allocate.argtypes = [VP]
        L.ref_pool_free.argtypes = [VP, I32]
        L.ref_pool_num_free.argtypes = [VP]
        L.ref_radix_create.argtypes = [VP]
        L.ref_radix_create.restype = VP
        L.ref_radix_destroy.argtypes = [VP]
        L.ref_radix_insert.argtypes = [VP, i32p, I32, i32p, I32]
        L.ref_radix_match.argtypes = [VP, i32p, I32, i32p, I32, C.POINTER(C.c_int)]
        L.ref_model_forward.argtypes = [I32] * 7 + [F32, F32] + [I32] * 5 + [VP, i32p, i32p, I32,
                                                                            f32p]
        L.ref_linear_create.argtypes = [VP, I32, I32]
        L.ref_linear_create.restype = VP
        L.ref_linear_run.argtypes = [VP, VP, I32, VP]
        L.ref_linear_destroy.argtypes = [VP]

    def embedding(self, w, ids):
        w, ids = _f(w), _i(ids)
        out = np.empty((ids.size, w.shape[1]), np.float32)
        self.lib.ref_embedding(w, w.shape[0], w.shape[1], ids, ids.size, out)
        return out

    def rmsnorm(self, x, w, eps):
        x, w = _f(x), _f(w)
        out = np.empty_like(x)
        self.lib.ref_rmsnorm(x, w, x.size // w.size, w.size, eps, out)
        return out

    def add_rmsnorm(self, x, residual, w, eps, first=False):
        x = _f(x).copy()
        r = np.empty_like(x) if first else _f(residual).copy()
        self.lib.ref_add_rmsnorm(x, r, _f(w), x.size // w.size, w.size, eps, int(first))
        return x, r

    def linear(self, x, w, out=None):
        x, w = _f(x), _f(w)
        N, K = w.shape
        T = x.size // K
        if out is None:
            out = np.empty((T, N), np.float32)
        self.lib.ref_linear(x.ctypes.data, w.ctypes.data, T, K, N, out.ctypes.data)
        return out

    def swiglu(self, g, u):
        g, u = _f(g), _f(u)
        out = np.empty_like(g)
        self.lib.ref_swiglu(g, u, g.size, out)
        return out

    def rope_table(self, head_dim, max_pos, base):
        t = np.empty((max_pos, head_dim), np.float32)
        self.lib.ref_rope_table(head_dim, max_pos, base, t)
        return t

    def rope(self, x, positions, num_heads, head_dim, max_pos, base):
        x = _f(x).copy()
        pos = _i(positions)
        self.lib.ref_rope(x, pos, pos.size, num_heads, head_dim, max_pos, base)
        return x

    def attention_mha(self, q, k, v, num_heads, head_dim):
        q, k, v = _f(q), _f(k), _f(v)
        out = np.empty_like(q)
        self.lib.ref_attention_mha(q, k, v, q.shape[0], num_heads, head_dim, out)
        return out

    def router(self, x, w, top_k, norm_topk=True):
        x, w = _f(x), _f(w)
        E, H = w.shape
        T = x.size // H
        ids = np.empty((T, top_k), np.int32)
        wts = np.empty((T, top_k), np.float32)
        self.lib.ref_router(x, w, T, H, E, top_k, int(norm_topk), ids, wts)
        return ids, wts

    def model_forward(self, cfg: dict, weights: list, ids, positions):
        arrs = [_f(w) for w in weights]
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        ids, positions = _i(ids), _i(positions)
        logits = np.empty((ids.size, cfg["vocab"]), np.float32)
        self.lib.ref_model_forward(
            cfg["num_layers"], cfg["hidden"], cfg["num_q_heads"], cfg["num_kv_heads"],
            cfg["head_dim"], cfg["inter"], cfg["vocab"], cfg["eps"], cfg["rope_base"], cfg.get("max_position", 64), cfg.get("num_experts", 0),
            cfg.get("top_k", 0), cfg.get("moe_inter", 0), int(cfg.get("norm_topk", True)),
            C.cast(ptrs, C.c_void_p), ids, positions, ids.size, logits)
        return logits


# ---- whole-layer / whole-model composition (src/model/qwen3.cpp:16-83, 168-180) ----
class _LayerT(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "input_ln", "w_qkv", "q_norm", "k_norm", "w_o", "post_ln", "w_gate_up", "w_down",
        "w_router", "expert_gate_up", "expert_down", "k_pool", "v_pool")]


class _ConfigT(C.Structure):
    _fields_ = [("hidden", C.c_int), ("num_q_heads", C.c_int), ("num_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("num_experts", C.c_int),
                ("top_k", C.c_int), ("moe_inter", C.c_int), ("norm_topk", C.c_int),
                ("eps", C.c_float), ("page_size", C.c_int)]


class _BatchT(C.Structure):
    _fields_ = [("num_tokens", C.c_int64), ("num_reqs", C.c_int), ("positions", C.c_void_p),
                ("slot_mapping", C.c_void_p), ("page_table", C.c_void_p), ("max_pages", C.c_int),
                ("seq_lens", C.c_void_p), ("q_indptr", C.c_void_p)]


class OracleModel:
    """fp32 model state for the oracle: weights (bf16-rounded values widened to fp32), per-layer
    paged K/V pools and the RoPE table. ``forward`` runs one scheduler step (qwen3.cpp:168-180)
    and returns the logits of each request's last token (fixes D10)."""

    def __init__(self, oracle: Oracle, cfg: dict, weights: dict, num_slots: int):
        self.o, self.cfg, self.w = oracle, cfg, {k: _f(v) for k, v in weights.items()}
        kd = cfg["num_kv_heads"] * cfg["head_dim"]
        L = cfg["num_layers"]
        self.k_pools = [np.zeros((num_slots, kd), np.float32) for _ in range(L)]
        self.v_pools = [np.zeros((num_slots, kd), np.float32) for _ in range(L)]
        self.table = oracle.rope_table(cfg["head_dim"], cfg["max_position"], cfg["rope_base"])
        self.lib = oracle.lib
        self.lib.oracle_decoder_layer.argtypes = [C.POINTER(_ConfigT), C.POINTER(_LayerT),
                                                  C.POINTER(_BatchT), f32p, f32p, f32p, C.c_int]
        c = cfg
        self.ct = _ConfigT(c["hidden"], c["num_q_heads"], c["num_kv_heads"], c["head_dim"],
                           c.get("inter", 0), c.get("num_experts", 0), c.get("top_k", 0),
                           c.get("moe_inter", 0), int(c.get("norm_topk", True)), c["eps"],
                           c["page_size"])
        self._keep = []
        self.layers = []
        for l in range(L):
            p = f"layers.{l}."
            g = lambda n: self.w[p + n].ctypes.data if (p + n) in self.w else None
            lt = _LayerT(g("input_ln"), g("qkv"), g("q_norm"), g("k_norm"), g("o"),
                         g("post_ln"), g("gate_up"), g("down"), g("router"), None, None,
                         self.k_pools[l].ctypes.data, self.v_pools[l].ctypes.data)
            E = c.get("num_experts", 0)
            if E:
                gu = (C.c_void_p * E)(*[self.w[p + f"experts.{e}.gate_up"].ctypes.data for e in range(E)])
                dn = (C.c_void_p * E)(*[self.w[p + f"experts.{e}.down"].ctypes.data for e in range(E)])
                self._keep += [gu, dn]
                lt.expert_gate_up = C.cast(gu, C.c_void_p)
                lt.expert_down = C.cast(dn, C.c_void_p)
            self.layers.append(lt)

    def forward(self, ids, positions, slot_mapping, page_table, seq_lens, q_indptr,
                return_hidden=False, return_state=False):
        """One step; `return_hidden`: also each layer's output x (the MLP output);
        `return_state`: also each layer's (x, residual) pair, whose fp32 sum residual + x is
        the hidden state after the layer."""
        c = self.cfg
        ids, positions, slots = _i(ids), _i(positions), _i(slot_mapping)
        pt, seq_lens, q_indptr = _i(page_table), _i(seq_lens), _i(q_indptr)
        T = ids.size
        bt = _BatchT(T, seq_lens.size, positions.ctypes.data, slots.ctypes.data, pt.ctypes.data,
                     pt.shape[1], seq_lens.ctypes.data, q_indptr.ctypes.data)
        x = self.o.embedding(self.w["embed"], ids)
        res = np.empty_like(x)
        hidden = []
        for l, lt in enumerate(self.layers):
            self.lib.oracle_decoder_layer(C.byref(self.ct), C.byref(lt), C.byref(bt), self.table,
                                          x, res, int(l == 0))
            if return_state:
                hidden.append((x.copy(), res.copy()))
            elif return_hidden:
                hidden.append(x.copy())
        last = q_indptr[1:] - 1
        xl, rl = x[last].copy(), res[last].copy()
        self.lib.oracle_add_rmsnorm(xl, rl, self.w["norm"], xl.shape[0], c["hidden"], c["eps"], 0)
        logits = self.o.linear(xl, self.w["lm_head"])
        return (logits, hidden) if (return_hidden or return_state) else logits
