"""Expert-parallel orchestration (nk_ep.ExpertParallelMoe) on 2 and 4 gloo ranks on
CPU, with the oracle as compute backend: sharding the experts over ranks and
exchanging routed rows must reproduce the single-process MoeLayer::forward_into
(moe.rs:154-249) on each rank's tokens bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, E, K, I, Is = 32, 8, 3, 16, 24


def _weights():
    r = np.random.default_rng(42)
    f = lambda *s: (r.standard_normal(s) * 0.3).astype(np.float32)  # noqa: E731
    return dict(router=f(H, E), up=f(E, H, I), down=f(E, I, H), sup=f(H, Is), sdown=f(Is, H))


def _worker(rank, world, port, tokens, mode, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, os.path.join(root, "nemotron-cutile-rs_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    import oracle as orc
    from ep_oracle_backend import OracleBackend
    from nk_ep import ExpertParallelMoe, local_expert_slice

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = _weights()
    be = OracleBackend(H, E, K, I, Is, mode, w["router"],
                       local_expert_slice(w["up"], rank, world, E),
                       local_expert_slice(w["down"], rank, world, E), w["sup"], w["sdown"])
    ep = ExpertParallelMoe(be, E, H, K)
    x = np.random.default_rng(100 + rank).standard_normal((tokens[rank], H)).astype(np.float32)
    out, idx, rw = ep.forward(torch.from_numpy(x))
    ref, ref_idx, ref_w = orc.moe(H, E, K, I, Is, w["router"], None, w["up"], None, w["down"],
                                  None, w["sup"], None, w["sdown"], None, x, tokens[rank], mode)
    q.put((rank, bool(np.array_equal(out.numpy().reshape(-1), ref)),
           bool(np.array_equal(idx.numpy(), ref_idx)), ep.last_exchange))
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("tokens,mode", [((37, 21), 0), ((5, 64), 2), ((1, 1), 1),
                                         ((9, 1, 30, 4), 2)])
def test_ep_ranks_match_single_process(tokens, mode):
    # 2 ranks (4 experts each) and 4 ranks (2 experts each, ragged token counts)
    world = len(tokens)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tokens, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same_out, same_idx, ex in sorted(results):
        assert same_idx, rank
        assert same_out, rank
        assert sum(ex["sent_rows"]) == tokens[rank] * K
