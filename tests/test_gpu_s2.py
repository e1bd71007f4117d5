"""The pack's planar S2 experts on the B200, bitwise against the oracle: the GGUF -> S2 re-layout, the Q8_0
activation rule (sgemv.mm:145-172 and its fp32-scale variant), the grouped decode API (moe_grouped_s2 over
moe_group_resident's groups, s2_expert_grouped.hpp:96-107), the hit path (moe_hit_select -> moe_hit_grouped_s2 ->
moe_hit_add, :80-91) and the streaming tier (the pack's expert file on disk -> ExpertCache slots -> the hit path)."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stratametal_b200 import api, synth

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def expert_rows(key, H, F):
    return (synth.quant_matrix(42, key, F, H, "cpu").numpy(), synth.quant_matrix(42, key + 1, F, H, "cpu").numpy(),
            synth.quant_matrix(42, key + 2, H, F, "cpu").numpy())


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("H,F", [(2560, 640), (2048, 512), (128, 64)])
def test_pack_equals_oracle(cuda, H, F):
    g, u, d = expert_rows(7, H, F)
    blob = torch.empty(api.s2_blob_bytes(H, F), dtype=torch.uint8, device=cuda)
    api.s2_pack_expert(dev(g, cuda), dev(u, cuda), dev(d, cuda), H, F, blob)
    assert np.array_equal(blob.cpu().numpy(), O.s2_pack(g, u, d, H, F))


@pytest.mark.parametrize("scaled", [False, True])
def test_quantize_q8_0(cuda, scaled):
    x = np.random.default_rng(5).standard_normal(4096).astype(np.float32)
    x[64:96] = 0.0
    x[100] = 3e4
    x[200:232] *= 1e-30
    y = torch.empty(4096 // 32 * 34, dtype=torch.uint8, device=cuda)
    s = torch.empty(4096 // 32, device=cuda) if scaled else None
    api.quantize_q8_0(dev(x, cuda), 4096, y, s)
    want = O.quant_q8_0(x, scaled)
    if scaled:
        assert np.array_equal(y.cpu().numpy(), want[0])
        assert np.array_equal(bits(s.cpu().numpy()), bits(want[1]))
    else:
        assert np.array_equal(y.cpu().numpy(), want)


def resident_arena(cuda, E, H, F, key=100):
    nb = api.s2_blob_bytes(H, F)
    host = [O.s2_pack(*expert_rows(key + 3 * e, H, F), H, F) for e in range(E)]
    return dev(np.concatenate(host), cuda), host, nb


@pytest.mark.parametrize("H,F,scaled", [(2560, 640, False), (2560, 640, True), (2048, 512, False)])
def test_grouped_resident_vs_oracle(cuda, H, F, scaled):
    E, T, k = 12, 3, 4
    arena, host, nb = resident_arena(cuda, E, H, F)
    rng = np.random.default_rng(H + F)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32).ravel()
    n = ids.size
    x = rng.standard_normal((T, H)).astype(np.float32)
    xq, xs = (O.quant_q8_0(x, True) if scaled else (O.quant_q8_0(x), None))
    grp_ptr = torch.empty(n, dtype=torch.int64, device=cuda)
    grp_start = torch.empty(n + 1, dtype=torch.int32, device=cuda)
    counts = torch.empty(2, dtype=torch.int32, device=cuda)
    ent_dst = torch.empty(n, dtype=torch.int32, device=cuda)
    ent_tok = torch.empty(n, dtype=torch.int32, device=cuda)
    api.moe_group_resident(dev(ids, cuda), n, k, arena.data_ptr(), nb, grp_ptr, grp_start, counts, ent_dst, ent_tok)
    torch.cuda.synchronize()
    # the groups: distinct ids ascending, entries in routing order
    distinct = np.unique(ids)
    ng = int(counts[0])
    assert ng == distinct.size and int(counts[1]) == n
    assert np.array_equal(grp_ptr.cpu().numpy()[:ng], arena.data_ptr() + distinct.astype(np.int64) * nb)
    order = np.argsort(ids, kind="stable")
    assert np.array_equal(ent_dst.cpu().numpy(), order)
    assert np.array_equal(ent_tok.cpu().numpy(), order // k)
    scratch = torch.empty(api.moe_grouped_scratch_bytes(n, H, F), dtype=torch.uint8, device=cuda)
    out = torch.full((n + 1, H), 7.0, device=cuda)
    api.device_status(clear=True)
    api.moe_grouped_s2(grp_ptr, grp_start, counts, ent_dst, ent_tok, n, n, H, F, dev(xq, cuda),
                       None if xs is None else dev(xs, cuda), scratch, out)
    torch.cuda.synchronize()
    assert api.device_status() == 0
    got = out.cpu().numpy()
    assert np.all(got[n] == 7.0), "wrote a row no entry names"
    nbx = H // 32
    for i in range(n):
        t = i // k
        want = O.s2_expert(host[ids[i]], H, F, xq[t * nbx * 34:(t + 1) * nbx * 34],
                           None if xs is None else xs[t * nbx:(t + 1) * nbx])
        assert np.array_equal(bits(got[i]), bits(want)), f"entry {i}"


def test_hits_streamed_from_the_pack(cuda, tmp_path):
    # experts stream from the pack on disk into a 5-slot VRAM tier; the routed ones that are resident run on the
    # hit path, the others keep the rows the caller left (the CPU tier's, in the reference's design)
    H, F, E, k = 2048, 512, 8, 6
    layers = [[O.s2_pack(*expert_rows(1000 * li + 3 * e, H, F), H, F) for e in range(E)] for li in range(2)]
    synth.write_native_pack(tmp_path, layers, 42, 42)
    nx = api.NativeExperts(tmp_path)
    nb = api.s2_blob_bytes(H, F)
    cache = api.ExpertCache(5, 2, E, nb)
    try:
        ids = np.array([6, 1, 3, 0, 7, 2], np.int32)
        for e in (1, 7, 4, 6, 2):
            p = nx.pick(1, e)
            assert p["blob_bytes"] == nb
            cache.ensure(1, e, p["host_blob"], nb)
        assert cache.ensure(1, 5, nx.pick(1, 5)["host_blob"], nb) == -1   # full: never evicts
        assert cache.slot_of(1, 7) == 1 and cache.slot_of(0, 7) == -1
        slot = torch.empty(k, dtype=torch.int32, device=cuda)
        dst = torch.empty(k, dtype=torch.int32, device=cuda)
        count = torch.empty(1, dtype=torch.int32, device=cuda)
        api.moe_hit_select(dev(ids, cuda), cache.row(1), k, E, slot, dst, count)
        torch.cuda.synchronize()
        hits = [i for i, e in enumerate(ids) if cache.slot_of(1, int(e)) >= 0]
        assert int(count[0]) == len(hits)
        assert np.array_equal(dst.cpu().numpy()[:len(hits)], hits)
        assert np.array_equal(slot.cpu().numpy()[:len(hits)], [cache.slot_of(1, int(ids[i])) for i in hits])
        x = np.random.default_rng(3).standard_normal(H).astype(np.float32)
        xq = O.quant_q8_0(x)
        scratch = torch.empty(api.moe_grouped_scratch_bytes(k, H, F), dtype=torch.uint8, device=cuda)
        out = torch.full((k, H), 7.0, device=cuda)
        api.device_status(clear=True)
        api.moe_hit_grouped_s2(cache.arena(), slot, dst, count, k, nb, H, F, dev(xq, cuda), None, 0, scratch, out)
        torch.cuda.synchronize()
        assert api.device_status() == 0
        got = out.cpu().numpy()
        for i in range(k):
            if i in hits:
                assert np.array_equal(bits(got[i]), bits(O.s2_expert(layers[1][ids[i]], H, F, xq))), f"hit {i}"
            else:
                assert np.all(got[i] == 7.0), f"miss {i} was written"
        # moe_hit_add: the hit rows added into parts the CPU tier filled elsewhere and left at zero here
        parts = torch.zeros(k, H, device=cuda)
        parts[[i for i in range(k) if i not in hits]] = 1.5
        api.moe_hit_add(parts, out, dst, count, k, H)
        torch.cuda.synchronize()
        pg = parts.cpu().numpy()
        for i in range(k):
            if i in hits:
                assert np.array_equal(bits(pg[i]), bits(got[i]))
            else:
                assert np.all(pg[i] == 1.5)
    finally:
        cache.close()
        nx.close()


def test_multi_token_hits(cuda):
    # a verify window: two tokens x k = 4 routed entries, each hit reading its own token's activation
    H, F, E, k, T = 2048, 512, 6, 4, 2
    arena, host, nb = resident_arena(cuda, E, H, F, key=500)
    ids = np.array([5, 0, 2, 3, 1, 4, 0, 5], np.int32)
    res = np.array([0, 1, -1, 3, -1, 5], np.int32)   # experts 2 and 4 are not resident
    slot = torch.empty(8, dtype=torch.int32, device=cuda)
    dst = torch.empty(8, dtype=torch.int32, device=cuda)
    count = torch.empty(1, dtype=torch.int32, device=cuda)
    res_d = dev(res, cuda)
    api.moe_hit_select(dev(ids, cuda), res_d.data_ptr(), 8, E, slot, dst, count)
    x = np.random.default_rng(9).standard_normal((T, H)).astype(np.float32)
    xq, xs = O.quant_q8_0(x, True)
    scratch = torch.empty(api.moe_grouped_scratch_bytes(8, H, F), dtype=torch.uint8, device=cuda)
    out = torch.full((8, H), 7.0, device=cuda)
    api.moe_hit_grouped_s2(arena.data_ptr(), slot, dst, count, 8, nb, H, F, dev(xq, cuda), dev(xs, cuda), k, scratch,
                           out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    nbx = H // 32
    for i, e in enumerate(ids):
        if res[e] < 0:
            assert np.all(got[i] == 7.0)
            continue
        t = i // k
        want = O.s2_expert(host[e], H, F, xq[t * nbx * 34:(t + 1) * nbx * 34], xs[t * nbx:(t + 1) * nbx])
        assert np.array_equal(bits(got[i]), bits(want)), f"entry {i}"
