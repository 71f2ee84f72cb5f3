"""The multi-GPU host logic on CPU: tile sharding of the crop loop and the
max-over-ranks timing rule, run as world-size-2 (and 3) gloo process groups
on 127.0.0.1, plus a rank that fails before a collective, which the others
must see as an error within the group's timeout rather than as a hang."""
import datetime
import os
import socket
import time

import pytest

from conftest import PKG_DIR

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")


def _mirror():
    import importlib.util
    spec = importlib.util.spec_from_file_location("sam3_b200_mp", os.path.join(PKG_DIR, "sam3_b200.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _shard_and_max(rank, world, port, total, out):
    dist = _init(rank, world, port, 60)
    sb = _mirror()
    start, count = sb.tile_shard(total, world, rank)
    blocks = [None] * world
    dist.all_gather_object(blocks, (start, count))
    elapsed = 10.0 + 3.0 * rank  # a per-rank "step time"
    slowest = sb.max_over_ranks(elapsed, dist)
    out.put((rank, blocks, slowest))
    dist.barrier()
    dist.destroy_process_group()


def _run(fn, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return results, [p.exitcode for p in procs]


def test_tile_shard_partitions_the_crop_loop():
    sb = _mirror()
    for total in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            blocks = [sb.tile_shard(total, world, r) for r in range(world)]
            covered = [i for s, c in blocks for i in range(s, s + c)]
            assert covered == list(range(total))
            counts = [c for _, c in blocks]
            assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        sb.tile_shard(64, 2, 2)


@pytest.mark.parametrize("world,total", [(2, 64), (3, 64)])
def test_gloo_ranks_shard_tiles_and_agree_on_the_slowest(world, total):
    results, codes = _run(_shard_and_max, world, _free_port(), total)
    assert codes == [0] * world
    for rank, blocks, slowest in results:
        assert sorted(blocks) == blocks  # contiguous blocks in rank order
        assert sum(c for _, c in blocks) == total
        assert slowest == 10.0 + 3.0 * (world - 1)


def _dies_before_barrier(rank, world, port, out):
    dist = _init(rank, world, port, 20)
    if rank == 1:
        out.put((rank, "left"))
        out.close()
        out.join_thread()  # the message is out before the process is
        os._exit(3)  # leaves between steps, no collective in flight
    t0 = time.time()
    try:
        dist.barrier()
        out.put((rank, "no error"))
    except Exception as e:  # the peer's socket closed, or the timeout expired
        out.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def test_gloo_rank_that_leaves_is_an_error_not_a_hang():
    results, codes = _run(_dies_before_barrier, 2, _free_port())
    msgs = dict(results)
    assert msgs[1] == "left"
    assert msgs[0].startswith("error after"), msgs[0]
    assert float(msgs[0].split()[2].rstrip("s:")) < 30.0
    assert codes[1] == 3
