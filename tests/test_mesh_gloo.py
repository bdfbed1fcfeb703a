"""Host logic of the column-sharded GEMM with 2 gloo ranks on CPU: the column
split, the rank order of exchanged IPC handles, the [P][M][N/P] -> row-major
re-layout, and a rank that dies before the gather turning into an error on the
other rank (not a hang)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_gather(rank, world, port, q):
    import sys
    sys.path[:0] = [os.environ["OJX_REPO"], os.path.join(os.environ["OJX_REPO"], "ojasx-open-source-cuda-_b200")]
    from torchcl.mesh import assemble_row_major, column_range, exchange_handles
    try:
        _init(rank, world, port)
        M, N, K = 6, 12, 5
        g = torch.Generator().manual_seed(0)
        A = torch.randn(M, K, generator=g)
        W = torch.randn(K, N, generator=g)
        bias = torch.randn(N, generator=g)
        c0, c1 = column_range(N, world, rank)
        local = torch.relu(A @ W[:, c0:c1] + bias[c0:c1])
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        gathered = torch.cat([p.reshape(-1) for p in parts])
        C = assemble_row_major(gathered, world, M, c1 - c0)
        ok = torch.allclose(C, torch.relu(A @ W + bias))
        handles = exchange_handles(bytes([rank]) * 64)
        ok = ok and [h[0] for h in handles] == list(range(world))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok))
    except Exception as e:  # report, never hang
        q.put((rank, repr(e)))


def _worker_dead_rank(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            os._exit(3)  # leaves before the gather, between steps (exit code checked)
        t = torch.ones(4)
        parts = [torch.empty(4) for _ in range(world)]
        try:
            dist.all_gather(parts, t)
            q.put((rank, "no error"))
        except Exception as e:
            q.put((rank, "error:" + type(e).__name__))
    except Exception as e:
        q.put((rank, "setup:" + repr(e)))


def _run(fn, world=2, timeout=120, expect=None):
    os.environ["OJX_REPO"] = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world if expect is None else expect):
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    out["exitcodes"] = [p.exitcode for p in procs]
    return out


def test_sharded_gather_host_logic():
    out = _run(_worker_gather)
    assert out[0] is True and out[1] is True, out


def test_dead_rank_becomes_an_error():
    out = _run(_worker_dead_rank, expect=1, timeout=90)
    assert out["exitcodes"][1] == 3
    assert out[0].startswith("error:"), out


def test_column_range_rules():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "ojasx-open-source-cuda-_b200"))
    from torchcl.mesh import column_range
    assert [column_range(32768, 8, r) for r in (0, 7)] == [(0, 4096), (28672, 32768)]
    with pytest.raises(ValueError):
        column_range(100, 8, 0)
    with pytest.raises(ValueError):
        column_range(64, 2, 2)


def test_should_shard_routes(monkeypatch):
    """Config 5 (32768^3) shards; config 4 decode shapes and config 3 on one rank
    stay whole; an uneven column split never shards; the env threshold applies."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "ojasx-open-source-cuda-_b200"))
    from torchcl.mesh import should_shard
    monkeypatch.delenv("OJX_SHARD_MIN_FLOPS", raising=False)
    assert should_shard(32768, 32768, 32768, 8)
    assert should_shard(8192, 11008, 4096, 2)
    assert not should_shard(8192, 11008, 4096, 1)
    for m in (1, 4, 16):
        assert not should_shard(m, 14336, 4096, 8)
    assert not should_shard(512, 512, 512, 8)
    assert not should_shard(4096, 1000, 4096, 8)
    monkeypatch.setenv("OJX_SHARD_MIN_FLOPS", "1e8")
    assert should_shard(512, 512, 512, 8)
    assert not should_shard(512, 512, 512, 8, min_flops=1e12)
