"""Host side of the peer finish without a GPU: the block layout, the handle
exchange and pointer tables of PeerGroup over a world-size-2 gloo group (with a
fake CUDA IPC backend), the descriptors it builds for both modes, and the C-ABI's
rejection of bad peer descriptors before it touches a device."""
import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from glmaxx_b200 import abi
from glmaxx_b200.peer import PeerGroup, plan_layout, two_shot_pays

T, H = 64, 6144
BUFFERS = {"partial": ((T, H), torch.float32), "out": ((T, H), torch.float32),
           "next_bf16": ((T, H), torch.bfloat16), "norm": ((T, H), torch.bfloat16)}


def test_layout_is_aligned_and_deterministic():
    a, sig, total = plan_layout(BUFFERS, 4)
    b, _, _ = plan_layout(dict(BUFFERS), 4)
    assert a == b and sig == 256
    assert all(s.offset % 256 == 0 for s in a.values())
    assert a["partial"].offset == 256
    assert a["out"].offset == 256 + T * H * 4
    assert total == 256 + 2 * T * H * 4 + 2 * T * H * 2
    with pytest.raises(ValueError):
        plan_layout(BUFFERS, 9)


def test_two_shot_threshold():
    assert not two_shot_pays(T * H, 2)
    assert two_shot_pays(2048 * H, 2)
    assert two_shot_pays(T * H, 8) and two_shot_pays(T * H, 4)
    assert not two_shot_pays(1024, 8) and not two_shot_pays(T * H, 1)


class FakeIpc:
    """Per-process fake: allocation returns a rank-specific address; a handle
    names the owner; open maps it at a fixed offset so tables are checkable."""

    def __init__(self, rank):
        self.rank = rank
        self.events = []

    def alloc(self, n):
        self.events.append(("alloc", n))
        return 0x7f0000000000 + self.rank * 0x100000000

    def handle(self, ptr):
        return ptr.to_bytes(8, "little") + bytes(56)

    def open(self, h):
        owner = int.from_bytes(h[:8], "little")
        self.events.append(("open", owner))
        return owner + 0x10000000000  # this process's mapping of the owner's block

    def close(self, ptr):
        self.events.append(("close", ptr))

    def free(self, ptr):
        self.events.append(("free", ptr))

    def zero(self, ptr, n):
        self.events.append(("zero", ptr, n))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake = FakeIpc(rank)
        g = PeerGroup(BUFFERS, backend=fake)
        res = {"bases": g.bases, "events": list(fake.events)}
        d, p = g.finish_descriptors("partial", out_f32="out", out_bf16="next_bf16",
                                    norm_bf16="norm", hidden=H, mode="two")
        arr = lambda a: list((ctypes.c_uint64 * world).from_address(a))  # noqa: E731
        res["partials"] = arr(d.partials_f32)
        res["signals"] = arr(p.signals_u32)
        res["outs"] = arr(p.outputs_f32)
        res["norms"] = arr(p.norms_bf16)
        res["flags"] = p.flags
        res["own_out"] = d.output_f32
        d1, p1 = g.finish_descriptors("partial", out_f32="out", mode="one")
        res["one"] = (p1.flags, p1.outputs_f32, d1.elements)
        # a token chunk: rows 16..48 of every buffer
        d2, p2 = g.finish_descriptors("partial", out_f32="out", norm_bf16="norm", hidden=H,
                                      mode="two", rows=(16, 48), row_elems=H)
        res["chunk"] = (d2.elements, arr(d2.partials_f32), arr(p2.outputs_f32),
                        arr(p2.norms_bf16), d2.output_f32)
        with pytest.raises(ValueError):
            g.finish_descriptors("partial", out_f32="out", rows=(60, 72), row_elems=H)
        with pytest.raises(ValueError):
            g.finish_descriptors("partial", out_f32=torch.empty(1), mode="two")
        g.close()
        res["closed"] = [e for e in fake.events if e[0] in ("close", "free")]
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_peer_group_two_ranks_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    slots, sig, total = plan_layout(BUFFERS, world)
    own = [0x7f0000000000 + r * 0x100000000 for r in range(world)]
    for r in range(world):
        res = results[r]
        expect = [own[p] if p == r else own[p] + 0x10000000000 for p in range(world)]
        assert res["bases"] == expect
        assert res["events"][0] == ("alloc", total)
        assert ("zero", own[r], sig) in res["events"]
        assert res["signals"] == expect
        assert res["partials"] == [b + slots["partial"].offset for b in expect]
        assert res["outs"] == [b + slots["out"].offset for b in expect]
        assert res["norms"] == [b + slots["norm"].offset for b in expect]
        assert res["own_out"] == res["outs"][r]
        assert res["flags"] == abi.PEER_TWO_SHOT
        assert res["one"] == (abi.PEER_ONE_SHOT, 0, T * H)
        assert res["closed"] == [("close", expect[1 - r]), ("free", own[r])]
        elements, parts, outs, norms, own_out = res["chunk"]
        assert elements == 32 * H
        assert parts == [b + slots["partial"].offset + 16 * H * 4 for b in expect]
        assert outs == [b + slots["out"].offset + 16 * H * 4 for b in expect]
        assert norms == [b + slots["norm"].offset + 16 * H * 2 for b in expect]
        assert own_out == outs[r]


def test_peer_launch_rejects_bad_descriptors_without_a_device():
    L = abi.load()
    s = ctypes.c_void_p(1)
    parts = (ctypes.c_uint64 * 2)(0x100000, 0x200000)
    sigs = (ctypes.c_uint64 * 2)(0x300000, 0x400000)
    outs = (ctypes.c_uint64 * 2)(0x500000, 0x600000)

    def descs(**pk):
        d = abi.MoeFinishDescriptor.new(abi_version=1, ranks=2, elements=4096,
                                        partials_f32=ctypes.addressof(parts),
                                        output_f32=0x500000)
        kw = dict(abi_version=1, flags=abi.PEER_ONE_SHOT, rank=0,
                  signals_u32=ctypes.addressof(sigs))
        kw.update(pk)
        return d, abi.MoePeerDescriptor.new(**kw)

    call = lambda d, p: L.glmaxx_moe_finish_peer_launch(  # noqa: E731
        ctypes.byref(d), ctypes.byref(p), s)
    assert L.glmaxx_moe_finish_peer_launch(None, None, s) == -1
    assert call(*descs(abi_version=2)) == -2
    assert call(*descs(flags=0)) == -2
    assert call(*descs(flags=3)) == -2
    assert call(*descs(rank=2)) == -2
    assert call(*descs(signals_u32=0)) == -1
    # one-shot takes no output arrays; two-shot needs them, with this rank's entry
    assert call(*descs(outputs_f32=ctypes.addressof(outs))) == -2
    assert call(*descs(flags=abi.PEER_TWO_SHOT)) == -1
    assert call(*descs(flags=abi.PEER_TWO_SHOT, rank=1, outputs_f32=ctypes.addressof(outs))) == -2
    d, p = descs(reserved=(ctypes.c_uint64 * 3)(0, 1, 0))
    assert call(d, p) == -2
    # the local finish still requires a residual
    d, _ = descs()
    assert L.glmaxx_moe_finish_launch(ctypes.byref(d), s) == -2
    assert L.glmaxx_moe_peer_signal_bytes(8) == 256 and L.glmaxx_moe_peer_signal_bytes(9) == 0
