"""msgl_paged_attention_decode_noalloc: decode on the library's static 8 MiB scratch.

Collected last (file name) so that it runs both after every other test in the session and, when
run on its own, in a fresh process. The no-allocation entry point must give exactly the bits of
msgl_paged_attention_decode with a caller workspace (it runs the same kernel), on two calls in a
row (the shared scratch keeps the previous call's partials and counters), and must reject a batch
whose scratch need exceeds 8 MiB without launching anything.
"""
import numpy as np
import pytest
import torch

from oracle import bf16_round

pytestmark = pytest.mark.gpu

P, D = 16, 128


def _bf16(rng, *shape):
    return bf16_round(rng.standard_normal(shape).astype(np.float32))


def _dev(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype).contiguous()


def _case(seed, seq_lens, hq, hkv):
    rng = np.random.default_rng(seed)
    pages_per = [(s + P - 1) // P for s in seq_lens]
    num_pages = sum(pages_per) + 5
    perm = rng.permutation(num_pages).astype(np.int32)
    pt = np.zeros((len(seq_lens), max(pages_per)), np.int32)
    off = 0
    for r, n in enumerate(pages_per):
        pt[r, :n] = perm[off:off + n]
        off += n
    kp = _dev(_bf16(rng, num_pages * P, hkv * D))
    vp = _dev(_bf16(rng, num_pages * P, hkv * D))
    q = _dev(_bf16(rng, len(seq_lens), hq * D))
    return q, kp, vp, _dev(pt, torch.int32), _dev(np.array(seq_lens, np.int32), torch.int32)


@pytest.mark.parametrize("seq_lens,hq,hkv", [
    ([300, 2048, 17, 777, 1], 32, 8),   # split-KV: the scratch holds partials and counters
    ([64, 5], 8, 8),                    # single chunk: no scratch use
    ([1000, 400, 2500], 16, 2),
])
def test_noalloc_matches_workspace_entry_point(cuda, seq_lens, hq, hkv):
    from msgl import ops
    q, kp, vp, pt, seq = _case(sum(seq_lens) + hq, seq_lens, hq, hkv)
    L = max(seq_lens)
    ref = ops.paged_attention_decode(q, kp, vp, pt, seq, L, hq, hkv)
    torch.cuda.synchronize()
    for _ in range(2):  # two calls in a row on the shared scratch
        out = ops.paged_attention_decode_noalloc(q, kp, vp, pt, seq, L, hq, hkv)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert ops.device_error() == (0, 0)


def test_noalloc_allocates_nothing_and_matches_oracle(cuda, oracle):
    """After a first call (which looks up the scratch address on this device), further calls with
    a preallocated output leave the device's free memory unchanged, and their output equals the
    oracle's fp32 paged attention within the per-op bf16 tolerance."""
    from msgl import ops
    seq_lens, hq, hkv = [300, 2048, 17, 777, 1], 32, 8
    q, kp, vp, pt, seq = _case(11, seq_lens, hq, hkv)
    L = max(seq_lens)
    out = torch.empty(len(seq_lens), hq, D, dtype=torch.bfloat16, device="cuda")
    ops.paged_attention_decode_noalloc(q, kp, vp, pt, seq, L, hq, hkv, out=out)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        ops.paged_attention_decode_noalloc(q, kp, vp, pt, seq, L, hq, hkv, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    B = len(seq_lens)
    ref = oracle.paged_attention(q.float().cpu().numpy().reshape(B, hq * D),
                                 kp.float().cpu().numpy(), vp.float().cpu().numpy(),
                                 pt.cpu().numpy(), seq.cpu().numpy(), np.arange(B + 1), hq, hkv,
                                 D, P)
    got = out.float().cpu().numpy().reshape(B, hq * D)
    err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert err < 1e-2, err
    assert ops.device_error() == (0, 0)


def test_noalloc_rejects_oversized_batch(cuda):
    from msgl import ops
    from msgl._lib import MsglError, lib
    hq, hkv, B, L = 64, 8, 512, 32768
    need = lib().msgl_paged_attention_workspace_size(B, L, hq, hkv, D)
    assert need > (8 << 20)
    q = torch.zeros(B, hq * D, dtype=torch.bfloat16, device="cuda")
    kp = torch.zeros(16 * P, hkv * D, dtype=torch.bfloat16, device="cuda")
    pt = torch.zeros(B, L // P, dtype=torch.int32, device="cuda")
    seq = torch.full((B,), L, dtype=torch.int32, device="cuda")
    with pytest.raises(MsglError) as e:
        ops.paged_attention_decode_noalloc(q, kp, kp, pt, seq, L, hq, hkv)
    assert e.value.code == 7  # MSGL_ERR_WORKSPACE
    assert ops.device_error() == (0, 0)


def test_attention_entry_points_on_two_devices_in_one_process(cuda):
    """One process drives two GPUs: decode, cascade decode, extend (tcgen05) and the no-allocation
    decode run on device 0 and then on device 1 (each device gets its own shared-memory opt-in and
    its own static scratch address); every output on device 1 equals device 0's bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from msgl import ops
    seq_lens, hq, hkv = [300, 2048, 17, 777, 1], 32, 8
    outs = []
    for d in (0, 1):
        with torch.cuda.device(d):
            q, kp, vp, pt, seq = _case(31, seq_lens, hq, hkv)
            L = max(seq_lens)
            r = [ops.paged_attention_decode(q, kp, vp, pt, seq, L, hq, hkv),
                 ops.paged_attention_decode_noalloc(q, kp, vp, pt, seq, L, hq, hkv)]
            # cascade: every request shares the first two pages of request 1's table
            shared = pt.clone()
            shared[:, :2] = pt[1, :2]
            seq_c = torch.clamp(seq, min=2 * P + 1)
            r.append(ops.paged_attention_decode_cascade(q, kp, vp, shared, seq_c, L, 2, hq, hkv))
            # extend: request 1 as a 256-token chunk at the end of its context
            qe = q.new_zeros(256, hq * D)
            qe.copy_(torch.randn(256, hq * D, generator=torch.Generator().manual_seed(5)).to(qe.dtype))
            ind = torch.tensor([0, 256], dtype=torch.int32, device=q.device)
            r.append(ops.paged_attention_extend(qe, kp, vp, pt[1:2].contiguous(), seq[1:2].contiguous(),
                                                ind, 256, hq, hkv))
            torch.cuda.synchronize()
            assert ops.device_error() == (0, 0)
            outs.append([x.cpu() for x in r])
    for a, b in zip(*outs):
        assert torch.equal(a, b)
