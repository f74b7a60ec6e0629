"""Tensor parallelism, host side, without a GPU: the argument checks every rank runs before it touches a device or
waits for the group, and the process plumbing of one process per GPU (group id exchange, max over ranks) on a
world-size-2 gloo group."""
import ctypes as C
import os
import socket

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _open_synth(wl, spec, **opt):
    h = C.c_void_p()
    o = wl.options(**opt)
    st = wl.lib().wl_open_synthetic(C.byref(spec), C.byref(o), C.byref(h))
    return st, wl.lib().wl_last_error().decode()


def test_options_carry_the_group(wl):
    gid = bytes(range(128))
    o = wl.options(tp_size=4, tp_rank=3, tp_id=gid)
    assert o.tp_size == 4 and o.tp_rank == 3 and bytes(o.tp_id) == gid
    d = wl.options()
    assert d.tp_size == 1 and d.tp_rank == 0


def test_unique_id_is_fresh(wl):
    a, b = wl.tp_unique_id(), wl.tp_unique_id()
    assert len(a) == 128 and len(b) == 128 and a != b


@pytest.mark.parametrize("case", ["rank", "heads", "moe", "vocab"])
def test_split_checks_fail_before_any_device_work(wl, case):
    from windlass_b200.transformer import config0_spec, synth_spec
    if case == "rank":        # rank outside 0..tp_size-1
        st, msg = _open_synth(wl, config0_spec(), tp_size=2, tp_rank=2)
        assert st == wl.WL_EINVAL and "tp_rank" in msg
    elif case == "heads":     # 8 heads do not split over 3 GPUs
        st, msg = _open_synth(wl, config0_spec(), tp_size=3, tp_rank=0)
        assert st == wl.WL_EUNSUPPORTED and "divisible by 3" in msg
    elif case == "moe":       # whole experts per GPU: 6 experts do not split over 4 GPUs
        st, msg = _open_synth(wl, synth_spec("qwen3moe", 1, 1024, 16, 8, 128, 0, 8192, experts=6, experts_used=2,
                                             expert_ff=512), tp_size=4, tp_rank=1)
        assert st == wl.WL_EUNSUPPORTED and "6 experts" in msg
    else:                     # a vocabulary too small for the ranks
        st, msg = _open_synth(wl, synth_spec("llama", 1, 2048, 32, 8, 64, 2048, 5), tp_size=8, tp_rank=0)
        assert st == wl.WL_EUNSUPPORTED and "vocabulary" in msg


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from windlass_b200 import tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gid = tp.share_group_id(dist)                       # rank 0 makes it with wl_tp_unique_id
        top = tp.max_over_ranks(dist, 10.0 + rank)
        q.put((rank, gid, top))
    finally:
        dist.destroy_process_group()


def test_group_id_and_max_over_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort()
    assert got[0][1] == got[1][1] and len(got[0][1]) == 128, "every rank must hold rank 0's group id"
    assert got[0][2] == got[1][2] == 11.0
