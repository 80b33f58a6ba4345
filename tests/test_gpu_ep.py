"""Expert parallelism on 2 B200s (NCCL over NVLink): each rank owns half of the
experts, routes its own tokens and exchanges routed rows.  The result must
match the single-GPU nk_moe_forward of the same tokens with all experts:
routing indices bit-exact, outputs within the bf16 bar (2e-2).  Skipped when
fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, E, K, I, Is, T = 512, 16, 4, 256, 384, 700


def _worker(rank, world, port, q, peer):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path.insert(0, os.path.join(root, "nemotron-cutile-rs_b200"))
    import torch.distributed as dist

    import nk
    from nk_ep import ExpertParallelMoe, NkBackend, PeerExpertParallelMoe, local_expert_slice

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    rn = lambda *s: torch.randn(*s, device=dev, generator=g) * 0.02  # noqa: E731
    router = rn(E, H)
    full = nk.MoeWeights(hidden=H, experts=E, top_k=K, inter=I, shared_inter=Is,
                         route_mode=nk.ROUTE_SIGMOID_RENORM, weight_kind=nk.W_BF16,
                         router_w3=nk.router_split(router), up_w=rn(E, I, H).bfloat16(),
                         down_w=rn(E, H, I).bfloat16(), shared_up_w=rn(Is, H).bfloat16(),
                         shared_down_w=rn(H, Is).bfloat16())
    local = nk.MoeWeights(hidden=H, experts=E // world, top_k=1, inter=I, shared_inter=0,
                          route_mode=full.route_mode, weight_kind=nk.W_BF16,
                          router_w3=full.router_w3,
                          up_w=local_expert_slice(full.up_w, rank, world, E),
                          down_w=local_expert_slice(full.down_w, rank, world, E))
    be = NkBackend(full, local)
    ep = (PeerExpertParallelMoe(be, E, H, K, max_tokens=T + 37 * world, phases=peer) if peer
          else ExpertParallelMoe(be, E, H, K))
    xg = torch.Generator(device=dev).manual_seed(10 + rank)
    x = torch.randn(T + 37 * rank, H, device=dev, generator=xg).bfloat16()
    out, idx, _ = ep.forward(x)
    out2, _, _ = ep.forward(x)  # buffers are reused across forwards
    assert torch.equal(out, out2)
    ref_idx = torch.empty_like(idx)
    ref = nk.MoeLayer(full).forward(x, indices=ref_idx)
    nk.device_status()
    err = ((out - ref).abs().max() / ref.abs().max()).item()
    q.put((rank, bool(torch.equal(idx, ref_idx)), err))
    if peer:
        ep.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("peer", [0, 1, 2], ids=["nccl_all_to_all", "nvlink_peer_stores",
                                               "nvlink_peer_stores_2_phases"])
def test_expert_parallel_two_gpus_matches_single_gpu(peer):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, peer)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same_idx, err in res:
        assert same_idx, rank
        assert err <= 2e-2, (rank, err)
