"""CPU: bench.py's data-parallel aggregation on two gloo ranks.

Each rank of a data-parallel bench run times its own request group; the
whole-job figure is the tokens summed over ranks divided by the slowest
rank's time.  Two processes stand in for two GPUs here (gloo on 127.0.0.1)."""
import os
import socket
import sys

import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q) -> None:
    sys.path.insert(0, REPO)
    import datetime

    import torch.distributed as dist

    from bench import RankSync

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        sync = RankSync(dist, "cpu")
        sync.barrier()
        # rank r: (r + 1) seconds for 100 * (r + 1) tokens
        tokens, seconds, value = sync.throughput(float(rank + 1), 100.0 * (rank + 1))
        exact = sync.reduce(0.0 if rank == 0 else 1.0, "sum")  # one rank reports a mismatch
        q.put((rank, tokens, seconds, value, exact))
    finally:
        dist.destroy_process_group()


def test_rank_sync_sums_tokens_and_takes_the_slowest_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, tokens, seconds, value, exact in out:
        assert tokens == 300.0 and seconds == 2.0 and value == 150.0
        assert exact == 1.0


def test_rank_sync_single_process_is_identity():
    sys.path.insert(0, REPO)
    from bench import RankSync

    tokens, seconds, value = RankSync().throughput(2.0, 50.0)
    assert (tokens, seconds, value) == (50.0, 2.0, 25.0)
