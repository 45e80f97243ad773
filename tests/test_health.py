"""Rank liveness on gloo CPU ranks: failures are made on the host (a rank that
raises and posts a notice, a rank that exits without one, a rank that never
joins); the survivors must learn of it between steps."""
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import torch
    import torch.distributed as dist

    from mod_b200.parallel.health import Heartbeat, RankFailure

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    # generous limit: under a loaded CI box a beat thread can stall for a while
    hb = Heartbeat(rank, world, interval=0.1, timeout=3.0).start()
    x = torch.ones(4)
    dist.all_reduce(x)  # one healthy step for everyone
    hb.check()
    dist.barrier()  # every rank has passed its healthy check before the victim fails
    victim = world - 1
    if rank == victim:
        if mode == "raise":
            try:
                raise RuntimeError("injected step error")
            except RuntimeError as e:
                hb.mark_failed(str(e))
            q.put((rank, "posted"))
            return
        if mode == "exit":
            os._exit(0)  # leaves between steps, no notice: survivors see the beats stop
        if mode == "leave":
            hb.leave()
            q.put((rank, "left"))
            return
    t0 = time.time()
    while True:
        try:
            hb.check()
        except RankFailure as e:
            q.put((rank, (e.ranks, e.reasons[victim], round(time.time() - t0, 2))))
            break
        if time.time() - t0 > 20.0:
            q.put((rank, "not detected"))
            break
        time.sleep(0.05)
    hb.stop()
    survivors = world - 1
    hb.store.add("mb_test/done", 1)
    if rank == 0:  # the store lives in this process: keep it up until every survivor has read it
        t1 = time.time()
        while hb.store.add("mb_test/done", 0) < survivors and time.time() - t1 < 20:
            time.sleep(0.05)


@pytest.mark.parametrize("mode", ["raise", "exit", "leave"])
def test_survivors_detect_rank_loss(mode):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    expected = world if mode in ("raise", "leave") else world - 1   # an exiting rank reports nothing
    res = {}
    try:
        for _ in range(expected):
            r, v = q.get(timeout=60)
            res[r] = v
    finally:
        for p in ps:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert isinstance(res.get(r), tuple), res
        ranks, reason, _ = res[r]
        assert ranks == [2]
        if mode == "raise":
            assert "injected step error" in reason
        elif mode == "leave":
            assert reason == "left"
        else:
            assert "heartbeat" in reason
            assert res[r][2] < 15.0


def test_never_joined_rank_is_reported():
    import torch.distributed as dist

    from mod_b200.parallel.health import Heartbeat, RankFailure

    store = dist.TCPStore("127.0.0.1", _port(), 1, is_master=True, wait_for_workers=False)
    hb = Heartbeat(0, 2, store=store, interval=0.05, timeout=0.3).start()
    hb.check()  # the peer gets ``timeout`` from the first look
    time.sleep(0.5)
    with pytest.raises(RankFailure) as ei:
        hb.check()
    assert ei.value.ranks == [1] and "no heartbeat" in ei.value.reasons[1]
    hb.stop()


def test_heartbeat_rejects_short_timeout():
    from mod_b200.parallel.health import Heartbeat

    with pytest.raises(ValueError):
        Heartbeat(0, 2, store=object(), interval=1.0, timeout=1.5)
