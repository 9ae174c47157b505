"""Expert parallelism on two GPUs (NCCL): each rank holds half of the experts, runs their jobs
(umsx_moe_forward_jobs), exchanges the job outputs and combines its tokens; the result must equal
the single-GPU layer bit for bit, on the per-stage path (T = 5) and the tensor-core prefill path
(T = 80), on the current stream and on a stream of the caller's own.  Skipped on a box with
fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, tokens, q):
    try:
        import datetime
        import importlib

        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        import __graft_entry__ as ge
        pkg = ge.load_package()
        ep = importlib.import_module(pkg.__name__ + ".ep")
        from oracle.oracle import Oracle
        from tests.helpers import bits, small_config, x_bits
        cfg = small_config()
        xb = x_bits(Oracle(), cfg, tokens)
        x = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).cuda(rank)
        full = pkg.MoeLayer(cfg.desc(tokens), synthetic=cfg.synthetic(), device=rank, reserve_bytes=1 << 28)
        want = full.forward(x).cpu().numpy()
        part = pkg.MoeLayer(cfg.desc(tokens, ep_rank=rank, ep_world=world), synthetic=cfg.synthetic(), device=rank,
                            reserve_bytes=1 << 28)
        out, (t0, t1) = ep.ExpertParallelLayer(part).forward(x)
        torch.cuda.synchronize()
        ok = np.array_equal(bits(out.cpu().numpy()), bits(want[t0:t1]))
        # the same on a stream of its own: every step of the layer is ordered on it
        side = torch.cuda.Stream(device=rank)
        side.wait_stream(torch.cuda.current_stream(rank))
        out2, _ = ep.ExpertParallelLayer(part).forward(x, stream=side)
        side.synchronize()
        ok = ok and np.array_equal(bits(out2.cpu().numpy()), bits(want[t0:t1]))
        q.put((rank, ok, t0, t1))
        part.close()
        full.close()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e), -1, -1))


@pytest.mark.parametrize("tokens", [5, 80])
def test_two_gpu_expert_parallel_layer_bit_exact(tokens):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tokens, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    covered = 0
    for rank, ok, t0, t1 in sorted(results):
        assert ok is True, (rank, ok)
        covered += t1 - t0
    assert covered == tokens
