"""Device-side decode batch metadata (msgl_decode_advance) against the host BatchBuilder /
PagePool, which follow Scheduler::step's flatten (scheduler.cpp:83-106) and KVCachePool's LIFO
allocation (kvcache.cpp:21-28). Integer outputs: bit-exact, step after step, including page
boundary crossings; exhaustion and page-table overflow leave every array untouched."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ERR_BOUNDS, ERR_WORKSPACE = 6, 7


def host_decode_meta(reqs, pool, P, width):
    from msgl.model import BatchBuilder
    bb = BatchBuilder(pool, P)
    ids, pos, slots, seq = [], [], [], []
    for r in reqs:
        bb._ensure_pages(r, r.device_len)
        p = r.device_len - 1
        ids.append(r.input_ids[-1])
        pos.append(p)
        slots.append(r.pages[p // P] * P + p % P)
        seq.append(r.device_len)
    pt = np.zeros((len(reqs), width), np.int32)
    for i, r in enumerate(reqs):
        pt[i, :len(r.pages)] = r.pages
    return np.array(ids, np.int32), np.array(pos, np.int32), np.array(slots, np.int32), pt, \
        np.array(seq, np.int32)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).cuda()


@pytest.mark.parametrize("B,steps", [(37, 40), (1, 20), (1100, 18)])
def test_decode_advance_matches_host(cuda, B, steps):
    from msgl import ops
    from msgl.model import PagePool, Request
    P, width = 16, 8
    rng = np.random.default_rng(B)
    num_pages = B * width + 5
    pool = PagePool(num_pages)
    rng.shuffle(pool.free)
    # lengths on and around page boundaries, then random
    lens = [int(x) for x in rng.integers(1, 80, B)]
    lens[0] = 16
    if B > 3:
        lens[1], lens[2], lens[3] = 15, 17, 32
    reqs = [Request([int(t) for t in rng.integers(0, 1000, n)]) for n in lens]
    ids, pos, slots, pt, seq = host_decode_meta(reqs, pool, P, width)
    d = dict(ids=dev(ids), pos=dev(pos), slots=dev(slots), pt=dev(pt), seq=dev(seq))
    free = dev(np.array(pool.free + [0] * 4, np.int32))  # the stack's unused tail is never read
    top = dev(np.array([len(pool.free)], np.int32))
    for step in range(steps):
        nxt = rng.integers(0, 1000, B).astype(np.int32)
        for r, t in zip(reqs, nxt):  # host: the sampled token joins each request
            r.input_ids.append(int(t))
        ids, pos, slots, pt, seq = host_decode_meta(reqs, pool, P, width)
        ops.decode_advance(dev(nxt), d["ids"], d["pos"], d["slots"], d["pt"], d["seq"], free, top,
                           page_size=P)
        torch.cuda.synchronize()
        for name, want in (("ids", ids), ("pos", pos), ("slots", slots), ("pt", pt), ("seq", seq)):
            got = d[name].cpu().numpy()
            assert np.array_equal(got, want), (step, name)
        assert int(top.item()) == len(pool.free), step
    assert ops.device_error() == (0, 0)


def test_decode_advance_exhaustion_and_overflow(cuda):
    from msgl import ops
    P = 16
    # two requests about to enter a new page, one page left: nothing may change
    seq = dev([32, 16, 5])
    pt = dev([[3, 4, 0], [7, 0, 0], [9, 0, 0]])
    ids, pos, slots = dev([1, 2, 3]), dev([31, 15, 4]), dev([4 * 16 + 15, 7 * 16 + 15, 9 * 16 + 4])
    free, top = dev([11, 12]), dev([1])
    snap = [t.clone() for t in (seq, pt, ids, pos, slots, free, top)]
    ops.decode_advance(dev([5, 6, 7]), ids, pos, slots, pt, seq, free, top, page_size=P)
    torch.cuda.synchronize()
    assert ops.device_error() == (ERR_WORKSPACE, 700)
    for a, b in zip((seq, pt, ids, pos, slots, free, top), snap):
        assert torch.equal(a, b)
    # a page past the page-table width
    seq2, pt2 = dev([48]), dev([[1, 2, 3]])
    ids2, pos2, slots2 = dev([0]), dev([47]), dev([3 * 16 + 15])
    free2, top2 = dev([20, 21]), dev([2])
    snap = [t.clone() for t in (seq2, pt2, ids2, pos2, slots2, top2)]
    ops.decode_advance(dev([9]), ids2, pos2, slots2, pt2, seq2, free2, top2, page_size=P)
    torch.cuda.synchronize()
    assert ops.device_error() == (ERR_BOUNDS, 701)
    for a, b in zip((seq2, pt2, ids2, pos2, slots2, top2), snap):
        assert torch.equal(a, b)
    # enough pages: both new pages come off the top, first request first
    top[0] = 2
    ops.decode_advance(dev([5, 6, 7]), ids, pos, slots, pt, seq, free, top, page_size=P)
    torch.cuda.synchronize()
    assert ops.device_error() == (0, 0)
    assert pt.cpu().numpy().tolist() == [[3, 4, 12], [7, 11, 0], [9, 0, 0]]
    assert slots.cpu().numpy().tolist() == [12 * 16, 11 * 16, 9 * 16 + 5]
    assert seq.cpu().numpy().tolist() == [33, 17, 6] and int(top.item()) == 0


def test_device_driven_decode_loop_matches_host_loop(cuda):
    """Greedy decode driven on the device (forward, then msgl_decode_advance feeding the next
    step) against the host-built steps: the same tokens."""
    from msgl import ops
    from msgl.model import BatchBuilder, BatchT, PagePool, Qwen3Model, Request, StepBatch
    from test_model_gpu import CFG, weights
    w = weights(CFG, 2)
    model = Qwen3Model(CFG, max_tokens=64, max_reqs=4)
    model.set_weights(w)
    num_pages, width, steps = 24, 6, 6
    rng = np.random.default_rng(3)
    prompts = [[int(t) for t in rng.integers(0, CFG["vocab"], n)] for n in (14, 31, 7)]
    runs = []
    for mode in ("host", "device"):
        model.alloc_kv(num_pages)
        pool = PagePool(num_pages)
        reqs = [Request(list(p)) for p in prompts]
        bb = BatchBuilder(pool)
        sb = bb.build(reqs, decode=False, max_pages=width)
        nxt = model.forward(sb)
        toks = [nxt.cpu().numpy().tolist()]
        for r, t in zip(reqs, toks[0]):
            r.cached_len = r.device_len
            r.input_ids.append(int(t))
        if mode == "host":
            for _ in range(steps):
                sb = bb.build(reqs, decode=True, max_pages=width)
                nxt = model.forward(sb)
                toks.append(nxt.cpu().numpy().tolist())
                for r, t in zip(reqs, toks[-1]):
                    r.input_ids.append(int(t))
        else:
            sb = bb.build(reqs, decode=True, max_pages=width)  # the first decode step's metadata
            t = sb.tensors
            free = torch.tensor(pool.free + [0], dtype=torch.int32, device="cuda")
            top = torch.tensor([len(pool.free)], dtype=torch.int32, device="cuda")
            st = sb.struct
            st.max_seq_len = width * 16  # an upper bound, valid for every step
            st.shared_prefix_pages = 0
            for s in range(steps):
                nxt = model.forward(StepBatch(t, st, len(reqs)))
                toks.append(nxt.cpu().numpy().tolist())
                if s + 1 < steps:
                    ops.decode_advance(nxt, t["input_ids"], t["positions"], t["slot_mapping"],
                                       t["page_table"], t["seq_lens"], free, top)
        runs.append(toks)
    assert runs[0] == runs[1]
    assert ops.device_error() == (0, 0)


def test_decode_steps_matches_host_loop(cuda):
    """msgl_model_decode_steps (a captured graph per step and the device advance between steps,
    no host in between) gives the tokens of the host-driven loop, over page boundaries."""
    from msgl.model import BatchBuilder, PagePool, Qwen3Model, Request
    from test_model_gpu import CFG, weights
    w = weights(CFG, 4)
    model = Qwen3Model(CFG, max_tokens=128, max_reqs=4)  # the prefill has 84 tokens
    model.set_weights(w)
    num_pages, width, steps = 32, 6, 12
    rng = np.random.default_rng(6)
    prompts = [[int(t) for t in rng.integers(0, CFG["vocab"], n)] for n in (12, 29, 3, 40)]
    runs = []
    s = torch.cuda.Stream()
    for mode in ("host", "device"):
        model.alloc_kv(num_pages)
        pool = PagePool(num_pages)
        reqs = [Request(list(p)) for p in prompts]
        bb = BatchBuilder(pool)
        with torch.cuda.stream(s):
            nxt = model.forward(bb.build(reqs, decode=False, max_pages=width))
        torch.cuda.synchronize()
        for r, t in zip(reqs, nxt.cpu().numpy().tolist()):
            r.cached_len = r.device_len
            r.input_ids.append(int(t))
        toks = []
        if mode == "host":
            for _ in range(steps):
                with torch.cuda.stream(s):
                    nxt = model.forward(bb.build(reqs, decode=True, max_pages=width), graph=True)
                torch.cuda.synchronize()
                toks.append(nxt.cpu().numpy().tolist())
                for r, t in zip(reqs, toks[-1]):
                    r.input_ids.append(int(t))
        else:
            with torch.cuda.stream(s):
                sb = bb.build(reqs, decode=True, max_pages=width)
                free = torch.tensor(pool.free + [0], dtype=torch.int32, device="cuda")
                top = torch.tensor([len(pool.free)], dtype=torch.int32, device="cuda")
                log = model.decode_steps(sb, steps, free, top, graph=True)
            torch.cuda.synchronize()
            toks = log.cpu().numpy().tolist()
        runs.append(toks)
    assert runs[0] == runs[1]
    from msgl import ops
    assert ops.device_error() == (0, 0)


def _prefilled(model, prompts, num_pages, width):
    from msgl.model import BatchBuilder, PagePool, Request
    model.alloc_kv(num_pages)
    pool = PagePool(num_pages)
    reqs = [Request(list(p)) for p in prompts]
    bb = BatchBuilder(pool)
    nxt = model.forward(bb.build(reqs, decode=False, max_pages=width))
    torch.cuda.synchronize()
    for r, t in zip(reqs, nxt.cpu().numpy().tolist()):
        r.cached_len = r.device_len
        r.input_ids.append(int(t))
    return pool, reqs, bb


def test_decode_steps_stop_rules(cuda):
    """msgl_model_decode_steps_stop against the reference's finish rule replayed on the host:
    per request max_tokens (3 / 20 / 5 / 20 new tokens), a stop id that request 0 emits at
    step 2 (request 2 ignores it), -1 in the log once a request finished; the active requests'
    tokens equal those of the run without rules (held requests do not disturb them), and no page
    is taken for a request after it finished."""
    from msgl.model import Qwen3Model
    from test_model_gpu import CFG, weights
    w = weights(CFG, 12)
    model = Qwen3Model(CFG, max_tokens=128, max_reqs=4)
    model.set_weights(w)
    num_pages, width, steps = 40, 8, 16
    rng = np.random.default_rng(13)
    prompts = [[int(t) for t in rng.integers(0, CFG["vocab"], n)] for n in (10, 31, 17, 5)]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        pool, reqs, bb = _prefilled(model, prompts, num_pages, width)
        sb = bb.build(reqs, decode=True, max_pages=width)
        free = torch.tensor(pool.free + [0], dtype=torch.int32, device="cuda")
        top = torch.tensor([len(pool.free)], dtype=torch.int32, device="cuda")
        free_log = model.decode_steps(sb, steps, free, top, graph=True)
    torch.cuda.synchronize()
    free_run = free_log.cpu().numpy()
    stop_id = int(free_run[2, 0])
    max_new = [20, 3, 20, 5]
    ignore = [0, 0, 1, 0]
    with torch.cuda.stream(s):
        pool, reqs, bb = _prefilled(model, prompts, num_pages, width)
        sb = bb.build(reqs, decode=True, max_pages=width)
        free = torch.tensor(pool.free + [0], dtype=torch.int32, device="cuda")
        top = torch.tensor([len(pool.free)], dtype=torch.int32, device="cuda")
        log, fin, gen = model.decode_steps_stop(sb, steps, free, top, max_new, [stop_id],
                                                ignore_eos=ignore, graph=True)
    torch.cuda.synchronize()
    got = log.cpu().numpy()
    # the finish rule on the host, over the unrestricted run's tokens
    exp = np.full_like(free_run, -1)
    done, n = [False] * 4, [0] * 4
    for st in range(steps):
        for r in range(4):
            if done[r]:
                continue
            t = int(free_run[st, r])
            exp[st, r] = t
            n[r] += 1
            if n[r] >= max_new[r] or (not ignore[r] and t == stop_id):
                done[r] = True
    assert np.array_equal(got, exp), (got, exp)
    assert fin.cpu().numpy().tolist() == [int(d) for d in done]
    assert gen.cpu().numpy().tolist() == n
    # pages: a finished request's page-table row and length stop moving
    seq = sb.tensors["seq_lens"].cpu().numpy()
    for r in range(4):
        last = max(st for st in range(steps) if exp[st, r] >= 0)
        assert seq[r] == len(prompts[r]) + 1 + (last if done[r] else steps - 1), (r, seq[r], last)
    from msgl import ops
    assert ops.device_error() == (0, 0)


def test_step_host_async_overlap(cuda):
    """Overlap scheduling: decode step s + 1 is submitted (msgl_model_step_host_async, input ids
    taken on the device from step s) before the host waits for step s; the tokens equal those of
    the synchronous msgl_model_step_host loop."""
    import ctypes as C

    import msgl
    from msgl.model import (DECODE_TAIL_DETECT, SHARED_PREFIX_DETECT, STEP_TOKENS_FROM_PREV, BatchT,
                            Qwen3Model)
    from test_model_gpu import CFG, weights
    w = weights(CFG, 14)
    model = Qwen3Model(CFG, max_tokens=128, max_reqs=4)
    model.set_weights(w)
    L = msgl.lib()
    num_pages, width, steps = 40, 8, 10
    rng = np.random.default_rng(15)
    prompts = [[int(t) for t in rng.integers(0, CFG["vocab"], n)] for n in (12, 3, 40, 22)]
    s = torch.cuda.Stream()
    sp = s.cuda_stream

    def host_batch(sb):
        h = {k: torch.from_numpy(np.ascontiguousarray(v.cpu().numpy())).pin_memory()
             for k, v in sb.tensors.items()}
        st = sb.struct
        hb = BatchT(st.num_tokens, st.num_reqs, st.is_decode, st.max_pages, st.max_seq_len,
                    st.max_q_len, *[h[k].data_ptr() for k in ("input_ids", "positions",
                                                              "slot_mapping", "page_table",
                                                              "seq_lens", "q_indptr", "last_idx")],
                    SHARED_PREFIX_DETECT, DECODE_TAIL_DETECT)
        return h, hb

    runs = []
    for mode in ("sync", "async"):
        with torch.cuda.stream(s):
            pool, reqs, bb = _prefilled(model, prompts, num_pages, width)
        toks, keep, pending = [], [], []
        outs = [torch.empty(4, dtype=torch.int32).pin_memory() for _ in range(steps)]
        for st in range(steps):
            sb = bb.build(reqs, decode=True, device="cpu", max_pages=width)
            h, hb = host_batch(sb)
            keep.append((h, hb))
            if mode == "sync":
                msgl.check(L.msgl_model_step_host(model.h, C.addressof(hb), outs[st].data_ptr(), 1, sp))
                ids = outs[st].numpy().tolist()
            else:
                tk = C.c_uint64()
                flags = 1 | (STEP_TOKENS_FROM_PREV if st > 0 else 0)
                msgl.check(L.msgl_model_step_host_async(model.h, C.addressof(hb), outs[st].data_ptr(),
                                                        flags, sp, C.byref(tk)))
                pending.append(tk.value)
                if st > 0:  # the previous step's tokens reach the host while this one runs
                    msgl.check(L.msgl_model_step_wait(model.h, pending[st - 1]))
                    toks.append(outs[st - 1].numpy().tolist())
                ids = None
            if mode == "sync":
                toks.append(ids)
            # lengths advance on the host; the ids are only needed by the sync loop's next batch
            for r, t in zip(reqs, ids if ids is not None else [0] * 4):
                r.cached_len = r.device_len
                r.input_ids.append(int(t))
        if mode == "async":
            msgl.check(L.msgl_model_step_wait(model.h, pending[-1]))
            toks.append(outs[steps - 1].numpy().tolist())
        runs.append(toks)
    assert runs[0] == runs[1]
    from msgl import ops
    assert ops.device_error() == (0, 0)
