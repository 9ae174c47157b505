"""Expert parallelism, host side: the exchange plan and the all-to-all of job outputs, run as
gloo ranks on the CPU.  Each rank keeps only the job outputs of its own experts (the rows
umsx_moe_forward_jobs writes on a GPU; here the oracle's per-job outputs, the others poisoned
with NaN), exchanges them, combines its tokens in rank order and must reproduce the oracle's
single-device layer bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import bf16_bits_to_f32, bits, host_weights, oracle_desc, small_config, x_bits


def _ep_module():
    import importlib

    import __graft_entry__ as ge
    pkg = ge.load_package()
    return importlib.import_module(pkg.__name__ + ".ep")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _combine(y, w):
    """Rank-order sum from 0.0f with explicit float32 roundings (the reference's combine)."""
    out = np.zeros((y.shape[0], y.shape[2]), np.float32)
    for r in range(y.shape[1]):
        out = (out + (w[:, r:r + 1] * y[:, r, :]).astype(np.float32)).astype(np.float32)
    return out


def _worker(rank, world, port, tokens, cfg_over, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle.oracle import Oracle
        orc = Oracle()
        ep = _ep_module()
        cfg = small_config(**cfg_over)
        want = orc.moe_layer(oracle_desc(cfg), host_weights(orc, cfg), bf16_bits_to_f32(x_bits(orc, cfg, tokens)),
                             threads=2)
        K, H, E = cfg.top_k, cfg.hidden, cfg.experts
        y = want["y"].reshape(tokens, K, H).copy()
        y[(want["ids"] // (E // world)) != rank] = np.nan  # rows of other ranks' experts must never be read
        got, (t0, t1) = ep.exchange(torch.from_numpy(y), torch.from_numpy(want["ids"]), E)
        ok = np.array_equal(bits(_combine(got.numpy(), want["weights"][t0:t1])), bits(want["out"][t0:t1]))
        q.put((rank, ok, t0, t1))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), -1, -1))


@pytest.mark.parametrize("world,tokens,over", [(2, 7, {}), (2, 1, {}), (3, 10, dict(experts=12, top_k=3))])
def test_expert_parallel_exchange_matches_single_device(world, tokens, over):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tokens, over, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    covered = 0
    for rank, ok, t0, t1 in sorted(results):
        assert ok is True, (rank, ok)
        covered += t1 - t0
    assert covered == tokens


def test_exchange_plan_is_a_permutation():
    ep = _ep_module()
    rng = np.random.default_rng(3)
    T, K, E = 37, 4, 16
    ids = torch.from_numpy(np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32))
    for world in (1, 2, 4):
        sent, recv_total = [], 0
        for rank in range(world):
            s_jobs, s_sizes, r_jobs, r_sizes = ep.plan_exchange(ids, E, world, rank)
            assert sum(s_sizes) == len(s_jobs) and sum(r_sizes) == len(r_jobs)
            sent.append(s_jobs)
            t0, t1 = ep.token_range(T, world, rank)
            assert sorted(r_jobs.tolist()) == list(range(t0 * K, t1 * K))
            recv_total += len(r_jobs)
        assert sorted(torch.cat(sent).tolist()) == list(range(T * K)) and recv_total == T * K


def _loss_worker(rank, world, port, q):
    """Both ranks exchange once; then rank 1 dies between steps (no collective in flight) and rank
    0's next exchange must end in an error, not a hang."""
    import datetime
    import time
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
        ep = _ep_module()
        T, K, H, E = 6, 2, 8, 4
        ids = torch.tensor([[0, 2], [1, 3], [2, 0], [3, 1], [0, 1], [2, 3]], dtype=torch.int32)
        y = torch.full((T, K, H), float(rank))
        ep.exchange(y, ids, E)
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # the message is out before the process goes
            os._exit(0)  # the rank is lost between steps
        time.sleep(1.0)
        t0 = time.time()
        try:
            ep.exchange(y, ids, E)
            q.put((rank, "no error"))
        except Exception as exc:  # the expected outcome
            q.put((rank, f"raised after {time.time() - t0:.1f}s: {type(exc).__name__}"))
    except Exception as exc:
        q.put((rank, "setup failed: " + repr(exc)))


def test_rank_loss_between_steps_raises_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_loss_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("raised after"), results[0]
