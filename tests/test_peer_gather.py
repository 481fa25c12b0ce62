"""Result all-gather over peer memory (``vtnk_peer_gather``), two ranks on two
GPUs (skipped with fewer): the gathered records equal an NCCL all-gather of
the same results on repeated calls (both buffer halves), and a rank whose
peer does not take part sees its bounded wait run out (status 1) instead of
hanging.  The absent peer stays alive -- it just never pushes -- so no kernel
ever writes into freed memory."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist

    from rectokens_b200.distributed import PeerGather

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        n, L = 1000, 3
        pg = PeerGather(n, L, dev, wait_ns=50_000_000 if mode == "absent" else 0)
        out = "ok"
        if mode == "match":
            for call in range(5):
                g = torch.Generator(device=dev).manual_seed(100 * call + rank)
                ids = torch.randint(0, 1 << 30, (n, L), device=dev, generator=g)
                node = torch.randint(0, 1 << 24, (n,), device=dev, generator=g)
                logp = -torch.rand(n, device=dev, generator=g)
                pg.push(ids, logp, node)
                gi, gl, gn, st = pg.result()
                ref_i = [torch.empty_like(ids) for _ in range(world)]
                ref_l = [torch.empty_like(logp) for _ in range(world)]
                ref_n = [torch.empty_like(node) for _ in range(world)]
                dist.all_gather(ref_i, ids)
                dist.all_gather(ref_l, logp)
                dist.all_gather(ref_n, node)
                assert st == 0, st
                assert torch.equal(gi.long(), torch.stack(ref_i)), call
                assert torch.equal(gl, torch.stack(ref_l)), call
                assert torch.equal(gn.long(), torch.stack(ref_n)), call
                dist.barrier()
        else:  # rank 1 never pushes: rank 0's barrier wait must run out
            if rank == 0:
                pg.push(torch.zeros((n, L), dtype=torch.long, device=dev),
                        torch.zeros(n, device=dev), torch.zeros(n, dtype=torch.long, device=dev))
                torch.cuda.synchronize()
                out = f"status={pg.result()[3]}"
            dist.barrier()
        torch.cuda.synchronize()
        dist.barrier()
        pg.close()
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["match", "absent"])
def test_peer_gather_two_ranks(mode, cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    if mode == "match":
        assert got == {0: "ok", 1: "ok"}, got
    else:
        assert got[0] == "status=1", got
        assert got[1] == "ok", got
