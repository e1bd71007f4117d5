"""Host side of expert parallelism on CPU: expert ranges, the handle exchange over a gloo process group of two
ranks (with the library's allocation and IPC calls replaced by fakes: no GPU here), refusal of a group whose
ranks disagree, and a rank that fails before the exchange ending the others' set-up with an error instead of a
hang."""
import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp

from stratametal_b200 import ep, synth
from stratametal_b200._lib import SmoeError


def test_expert_ranges_partition_the_pool():
    for world in (1, 2, 4, 8):
        rs = [ep.expert_range(512, r, world) for r in range(world)]
        assert [e for r in rs for e in r] == list(range(512))
    with pytest.raises(SmoeError):
        ep.expert_range(500, 0, 8)
    with pytest.raises(SmoeError):
        ep.expert_range(512, 0, 9)
    with pytest.raises(SmoeError):
        ep.expert_range(512, 2, 2)


def test_shard_planes_are_the_pool_slices():
    spec = synth.LayerSpec(n_embd=128, n_ff=64, n_expert=8, k=2, seed=3)
    full = synth.make_layer(spec, 0)
    for r in range(2):
        sh = ep.shard_layer(spec, 0, r, 2, "cpu")
        for name in ("ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight"):
            n = sh[name].shape[0]
            assert (sh[name] == full[name][r * n:(r + 1) * n]).all()
        for name in ("ffn_gate_inp.weight", "ffn_gate_shexp.weight", "ffn_down_shexp.weight"):
            assert (sh[name] == full[name]).all()


class FakeLib:
    """Stands in for libsmoe.so's set-up calls: areas are integers, handles are bytes naming them."""

    def __init__(self, rank):
        self.rank, self.opened, self.closed, self.freed = rank, [], [], []

    def smoe_ep_area_bytes(self, c, max_tokens, world):
        return 4096 + max_tokens * world

    def smoe_ep_area_open(self, buf, ptr):
        src = bytes(buf)[0]
        ptr._obj.value = 0x100000 * (src + 1)
        self.opened.append(src)
        return 0

    def smoe_ep_area_close(self, a):
        self.closed.append(a.value)
        return 0

    def smoe_ep_area_free(self, a):
        self.freed.append(a.value)
        return 0


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        fake = FakeLib(rank)
        ep.lib = lambda: fake
        ep.EpAreas._alloc = staticmethod(
            lambda nbytes, want: (0x100000 * (rank + 1), bytes([rank]) + bytes(63)))
        spec = synth.LayerSpec(n_embd=512, n_ff=128, n_expert=16, k=4, seed=1)
        Tm = 8
        if mode == "mismatch" and rank == 1:
            Tm = 9
        if mode == "dies" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        a = ep.EpAreas.distributed(spec, Tm)
        d = a.desc()
        res = {"rank": d.rank, "world": d.world, "max_tokens": d.max_tokens,
               "areas": [d.areas[i] for i in range(world)], "opened": sorted(fake.opened)}
        a.close()
        res["closed"], res["freed"] = fake.closed, fake.freed
        q.put((rank, "ok", res))
    except Exception as e:
        q.put((rank, "error", type(e).__name__ + ": " + str(e)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, kind, val = q.get(timeout=120)
        out[r] = (kind, val)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_handle_exchange_two_ranks():
    out = _run("ok")
    for r in range(2):
        kind, res = out[r]
        assert kind == "ok", res
        assert res["rank"] == r and res["world"] == 2 and res["max_tokens"] == 8
        assert res["areas"] == [0x100000, 0x200000]       # rank order, own area at [rank]
        assert res["opened"] == [1 - r]                     # the other rank's handle, opened once
        assert res["closed"] == [0x100000 * (2 - r)] and res["freed"] == [0x100000 * (r + 1)]


def test_disagreeing_ranks_are_refused_everywhere():
    out = _run("mismatch")
    for r in range(2):
        kind, msg = out[r]
        assert kind == "error" and "disagree" in msg, msg


def test_rank_failing_before_exchange_ends_the_others_setup():
    out = _run("dies")
    assert out[1][0] == "error"
    assert out[0][0] == "error", "rank 0 must get an error (peer gone or timeout), not hang"
