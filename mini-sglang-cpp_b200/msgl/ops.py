"""torch-tensor front end of the libmsgl C ABI (device memory and streams come from torch).

Each function checks shapes / dtypes, then calls the matching ``msgl_*`` entry point on the
current torch stream. No function here computes anything itself.
"""
from __future__ import annotations

import torch

from ._lib import check, lib

BF16, F32 = 1, 0
_DT = {torch.bfloat16: BF16, torch.float32: F32}


def _s():
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _c(t, dtype=None):
    assert t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    if dtype is not None:
        assert t.dtype == dtype, f"expected {dtype}, got {t.dtype}"
    return t


# ------------------------------------------------------------------ reference launchers
def rmsnorm(x, w, eps):
    _c(x), _c(w, x.dtype)
    out = torch.empty_like(x)
    H = w.numel()
    check(lib().msgl_launch_rmsnorm(_p(x), _p(w), _p(out), x.numel() // H, H, eps, _DT[x.dtype], _s()))
    return out


def rope_(q, k, positions, cos_sin, num_q_heads, num_kv_heads, head_dim):
    """In-place rotate-half RoPE on q [T, Hq*D] and k [T, Hkv*D] (k may be None)."""
    _c(q), _c(positions, torch.int32), _c(cos_sin, torch.float32)
    check(lib().msgl_launch_rope(_p(q), _p(k), _p(positions), _p(cos_sin), positions.numel(),
                                 num_q_heads, num_kv_heads, head_dim, _DT[q.dtype], _s()))


def index_gather(table, ids):
    _c(table), _c(ids, torch.int32)
    out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    check(lib().msgl_launch_index_gather(_p(table), _p(ids), _p(out), table.shape[1], ids.numel(),
                                         table.shape[0], _DT[table.dtype], _s()))
    return out


def store_kv_page(k, v, k_cache, v_cache, page_table, page_size, num_heads, head_dim):
    _c(k), _c(v), _c(k_cache), _c(v_cache), _c(page_table, torch.int32)
    T = k.numel() // (num_heads * head_dim)
    check(lib().msgl_launch_store_kv_page(_p(k), _p(v), _p(k_cache), _p(v_cache), _p(page_table),
                                          page_size, num_heads, head_dim, T, _DT[k.dtype], _s()))


# ------------------------------------------------------------------ fused ops
def add_rmsnorm_(x, residual, w, eps, first=False):
    """In place: residual += x (or = x when first); x = rmsnorm(residual) * w."""
    _c(x, torch.bfloat16), _c(residual, torch.float32), _c(w, torch.bfloat16)
    H = w.numel()
    check(lib().msgl_add_rmsnorm(_p(x), _p(residual), _p(w), x.numel() // H, H, eps, int(first), _s()))


def add_partials_rmsnorm_(parts, x, residual, w, eps):
    """residual += sum_p parts[p] (fp32 split-K partials [P, T, H], added in p order);
    x = rmsnorm(residual) * w (x written in place)."""
    _c(parts, torch.float32), _c(x, torch.bfloat16), _c(residual, torch.float32), _c(w, torch.bfloat16)
    H = w.numel()
    T = x.numel() // H
    check(lib().msgl_add_partials_rmsnorm(_p(parts), parts.numel() // (T * H), _p(x), _p(residual),
                                          _p(w), T, H, eps, _s()))


def embed_rmsnorm(embed, ids, w, eps):
    _c(embed, torch.bfloat16), _c(ids, torch.int32), _c(w, torch.bfloat16)
    V, H = embed.shape
    x = torch.empty(ids.numel(), H, dtype=torch.bfloat16, device=embed.device)
    r = torch.empty(ids.numel(), H, dtype=torch.float32, device=embed.device)
    check(lib().msgl_embed_rmsnorm(_p(embed), _p(ids), ids.numel(), V, H, _p(w), eps, _p(x), _p(r), _s()))
    return x, r


def qknorm_rope_store_kv(qkv, k_pool, v_pool, positions, slot_mapping, cos_sin, q_norm, k_norm,
                         num_q_heads, num_kv_heads, eps, head_dim=128):
    _c(qkv, torch.bfloat16), _c(k_pool, torch.bfloat16), _c(v_pool, torch.bfloat16)
    _c(positions, torch.int32), _c(slot_mapping, torch.int32), _c(cos_sin, torch.float32)
    T = positions.numel()
    q = torch.empty(T, num_q_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    num_slots = k_pool.numel() // (num_kv_heads * head_dim)
    check(lib().msgl_qknorm_rope_store_kv(_p(qkv), _p(q), _p(k_pool), _p(v_pool), num_slots,
                                          _p(positions), _p(slot_mapping), _p(cos_sin), _p(q_norm),
                                          _p(k_norm), T, num_q_heads, num_kv_heads, head_dim, eps, _s()))
    return q


def qknorm_rope_store_kv_partials(parts, k_pool, v_pool, positions, slot_mapping, cos_sin, q_norm,
                                  k_norm, num_q_heads, num_kv_heads, eps, head_dim=128):
    """As qknorm_rope_store_kv with the QKV rows the sum of fp32 partials [P, T, (Hq+2Hkv) D]."""
    _c(parts, torch.float32), _c(k_pool, torch.bfloat16), _c(v_pool, torch.bfloat16)
    _c(positions, torch.int32), _c(slot_mapping, torch.int32), _c(cos_sin, torch.float32)
    T = positions.numel()
    nparts = parts.numel() // (T * (num_q_heads + 2 * num_kv_heads) * head_dim)
    q = torch.empty(T, num_q_heads, head_dim, dtype=torch.bfloat16, device=parts.device)
    num_slots = k_pool.numel() // (num_kv_heads * head_dim)
    check(lib().msgl_qknorm_rope_store_kv_partials(
        _p(parts), nparts, _p(q), _p(k_pool), _p(v_pool), num_slots, _p(positions),
        _p(slot_mapping), _p(cos_sin), _p(q_norm), _p(k_norm), T, num_q_heads, num_kv_heads,
        head_dim, eps, _s()))
    return q


def decode_advance(next_tokens, input_ids, positions, slot_mapping, page_table, seq_lens,
                   free_pages, free_top, page_size=16):
    """msgl_decode_advance on device int32 tensors (in place): the next decode step's metadata."""
    for t in (next_tokens, input_ids, positions, slot_mapping, page_table, seq_lens, free_pages,
              free_top):
        _c(t, torch.int32)
    B = seq_lens.numel()
    check(lib().msgl_decode_advance(_p(next_tokens), _p(input_ids), _p(positions),
                                    _p(slot_mapping), _p(page_table), page_table.shape[1],
                                    _p(seq_lens), _p(free_pages), _p(free_top), B, page_size, _s()))


def sample(logits, temperature, top_k, top_p, seed=0, step=0, out=None):
    """msgl_sample: one token id per row of fp32 logits [B, V] (per-row parameters, device)."""
    _c(logits, torch.float32), _c(temperature, torch.float32), _c(top_k, torch.int32)
    _c(top_p, torch.float32)
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    check(lib().msgl_sample(_p(logits), B, V, _p(temperature), _p(top_k), _p(top_p), seed, step,
                            _p(out), _s()))
    return out


# ------------------------------------------------------------------ attention
def attention_workspace(num_reqs, max_seq_len, hq, hkv, device="cuda"):
    n = lib().msgl_paged_attention_workspace_size(num_reqs, max_seq_len, hq, hkv, 128)
    return torch.zeros(max(n, 256), dtype=torch.uint8, device=device)


def paged_attention_decode(q, k_pool, v_pool, page_table, seq_lens, max_seq_len, hq, hkv,
                           scale=None, page_size=16, workspace=None, out=None):
    _c(q, torch.bfloat16), _c(page_table, torch.int32), _c(seq_lens, torch.int32)
    B = seq_lens.numel()
    if scale is None:
        scale = 1.0 / (128 ** 0.5)
    if workspace is None:
        workspace = attention_workspace(B, max_seq_len, hq, hkv, q.device)
    if out is None:
        out = torch.empty(B, hq, 128, dtype=torch.bfloat16, device=q.device)
    num_slots = k_pool.numel() // (hkv * 128)
    check(lib().msgl_paged_attention_decode(_p(q), _p(k_pool), _p(v_pool), num_slots,
                                            _p(page_table), page_table.shape[1], _p(seq_lens), B,
                                            max_seq_len, hq, hkv, 128, page_size, scale, _p(out),
                                            _p(workspace), workspace.numel(), _s()))
    return out


def paged_attention_decode_cascade(q, k_pool, v_pool, page_table, seq_lens, max_seq_len,
                                   shared_pages, hq, hkv, scale=None, page_size=16, workspace=None,
                                   out=None):
    """msgl_paged_attention_decode_cascade: decode with the first `shared_pages` page-table
    columns common to every request."""
    _c(q, torch.bfloat16), _c(page_table, torch.int32), _c(seq_lens, torch.int32)
    B = seq_lens.numel()
    if scale is None:
        scale = 1.0 / (128 ** 0.5)
    if workspace is None:
        n = lib().msgl_paged_attention_cascade_workspace_size(B, max_seq_len, shared_pages, hq, hkv, 128)
        workspace = torch.zeros(max(n, 256), dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty(B, hq, 128, dtype=torch.bfloat16, device=q.device)
    num_slots = k_pool.numel() // (hkv * 128)
    check(lib().msgl_paged_attention_decode_cascade(_p(q), _p(k_pool), _p(v_pool), num_slots,
                                                    _p(page_table), page_table.shape[1],
                                                    _p(seq_lens), B, max_seq_len, shared_pages, hq,
                                                    hkv, 128, page_size, scale, _p(out),
                                                    _p(workspace), workspace.numel(), _s()))
    return out


def paged_attention_decode_noalloc(q, k_pool, v_pool, page_table, seq_lens, max_seq_len, hq, hkv,
                                   scale=None, page_size=16, out=None):
    """msgl_paged_attention_decode_noalloc: decode on the library's static scratch."""
    _c(q, torch.bfloat16), _c(page_table, torch.int32), _c(seq_lens, torch.int32)
    B = seq_lens.numel()
    if scale is None:
        scale = 1.0 / (128 ** 0.5)
    if out is None:
        out = torch.empty(B, hq, 128, dtype=torch.bfloat16, device=q.device)
    num_slots = k_pool.numel() // (hkv * 128)
    check(lib().msgl_paged_attention_decode_noalloc(_p(q), _p(k_pool), _p(v_pool), num_slots,
                                                    _p(page_table), page_table.shape[1],
                                                    _p(seq_lens), B, max_seq_len, hq, hkv, 128,
                                                    page_size, scale, _p(out), _s()))
    return out


def paged_attention_extend(q, k_pool, v_pool, page_table, seq_lens, q_indptr, max_q_len, hq, hkv,
                           scale=None, page_size=16):
    _c(q, torch.bfloat16), _c(page_table, torch.int32), _c(seq_lens, torch.int32)
    _c(q_indptr, torch.int32)
    B = seq_lens.numel()
    if scale is None:
        scale = 1.0 / (128 ** 0.5)
    out = torch.zeros_like(q)
    num_slots = k_pool.numel() // (hkv * 128)
    check(lib().msgl_paged_attention_extend(_p(q), _p(k_pool), _p(v_pool), num_slots,
                                            _p(page_table), page_table.shape[1], _p(seq_lens),
                                            _p(q_indptr), B, max_q_len, hq, hkv, 128, page_size,
                                            scale, _p(out), _s()))
    return out


# ------------------------------------------------------------------ GEMMs
def gemm_workspace(M, N, K, device="cuda"):
    n = lib().msgl_gemm_workspace_size(M, N, K)
    return torch.zeros(max(n, 256), dtype=torch.uint8, device=device)


def linear(x, w, out_dtype=torch.bfloat16, workspace=None):
    """y = x W^T with W [N, K] (Linear::forward)."""
    _c(x, torch.bfloat16), _c(w, torch.bfloat16)
    N, K = w.shape
    M = x.numel() // K
    y = torch.empty(M, N, dtype=out_dtype, device=x.device)
    if workspace is None:
        workspace = gemm_workspace(M, N, K, x.device)
    check(lib().msgl_gemm_bf16(_p(x), _p(w), _p(y), M, N, K, _DT[out_dtype], _p(workspace),
                               workspace.numel(), _s()))
    return y


def gemm_partials_splits(M, N, K):
    return lib().msgl_gemm_partials_splits(M, N, K)


def linear_partials(x, w, splits=None, out=None):
    """fp32 split-K partials [S, M, N] of x W^T (sum over S = x W^T)."""
    _c(x, torch.bfloat16), _c(w, torch.bfloat16)
    N, K = w.shape
    M = x.numel() // K
    if splits is None:
        splits = gemm_partials_splits(M, N, K)
    if out is None:
        out = torch.empty(splits, M, N, dtype=torch.float32, device=x.device)
    check(lib().msgl_gemm_bf16_partials(_p(x), _p(w), _p(out), M, N, K, splits, _s()))
    return out


def pack_gate_up(w_gate_up):
    _c(w_gate_up, torch.bfloat16)
    two_i, K = w_gate_up.shape
    out = torch.empty_like(w_gate_up)
    check(lib().msgl_pack_gate_up(_p(w_gate_up), _p(out), two_i // 2, K, _s()))
    return out


def gate_up_silu(x, w_packed, workspace=None):
    _c(x, torch.bfloat16), _c(w_packed, torch.bfloat16)
    two_i, K = w_packed.shape
    M = x.numel() // K
    y = torch.empty(M, two_i // 2, dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = gemm_workspace(M, two_i, K, x.device)
    check(lib().msgl_gemm_gate_up_silu(_p(x), _p(w_packed), _p(y), M, two_i // 2, K, _p(workspace),
                                       workspace.numel(), _s()))
    return y


def lm_head_argmax(x, w, workspace=None):
    _c(x, torch.bfloat16), _c(w, torch.bfloat16)
    V, K = w.shape
    M = x.numel() // K
    packed = torch.empty(M, dtype=torch.int64, device=x.device)
    ids = torch.empty(M, dtype=torch.int32, device=x.device)
    if workspace is None:
        workspace = gemm_workspace(M, V, K, x.device)
    check(lib().msgl_lm_head_argmax(_p(x), _p(w), M, V, K, _p(packed), _p(ids), _p(workspace),
                                    workspace.numel(), _s()))
    return ids


def argmax(logits):
    _c(logits)
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    check(lib().msgl_argmax(_p(logits), logits.shape[0], logits.shape[1], _DT[logits.dtype], _p(out), _s()))
    return out


def fill_normal_(t, seed, stream_id=0, mean=0.0, std=1.0):
    _c(t, torch.bfloat16)
    check(lib().msgl_fill_normal_bf16(_p(t), t.numel(), seed, stream_id, mean, std, _s()))
    return t


def device_error(reset=True):
    import ctypes as C
    code, info = C.c_int(0), C.c_int(0)
    check(lib().msgl_device_error(C.addressof(code), C.addressof(info), int(reset), _s()))
    return code.value, info.value
