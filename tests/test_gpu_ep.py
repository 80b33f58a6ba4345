"""Expert parallelism on 2 B200s: each rank owns half of the experts, routes
its own tokens and exchanges routed rows with the other rank.  Every
exchange — the native C-ABI executor (nk_moe_forward_ep: counts, rows and
results moved by libnk kernels over NVLink peer memory, device barriers; rows
pulled by the owners' up projection or pushed before it), the
Python-orchestrated peer-store exchange and NCCL all-to-all-v — must
reproduce the oracle's MoeLayer::forward_into restatement (moe.rs:154-249) on
the rank's own tokens: routing indices bit-exact, outputs within the bf16 bar
(2e-2).  Ranks hold different token counts.  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, E, K, I, Is, T = 512, 16, 4, 256, 384, 700


def _worker(rank, world, port, q, mode):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in ("nemotron-cutile-rs_b200", "oracle"):
        sys.path.insert(0, os.path.join(root, p))
    import torch.distributed as dist

    import nk
    import oracle as orc
    from nk_ep import (ExpertParallelMoe, NativeExpertParallelMoe, NkBackend,
                       PeerExpertParallelMoe, local_layer)

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
    local = local_layer(full, rank, world)
    tmax = T + 37 * world
    if mode == "native_pull":  # rows pulled by the owners' up projection
        os.environ["NK_EP_PULL"] = "1"
    if mode.startswith("native"):
        ep = NativeExpertParallelMoe(full, local, max_tokens=tmax)
    else:
        be = NkBackend(full, local)
        ep = (PeerExpertParallelMoe(be, E, H, K, max_tokens=tmax, phases=2 if mode == "peer2"
                                    else 1) if mode.startswith("peer")
              else ExpertParallelMoe(be, E, H, K))
    xg = torch.Generator(device=dev).manual_seed(10 + rank)
    x = torch.randn(T + 37 * rank, H, device=dev, generator=xg).bfloat16()
    out, idx, _ = ep.forward(x)
    out2, _, _ = ep.forward(x)  # buffers are reused across forwards
    same_repeat = bool(torch.equal(out, out2))
    nk.device_status()
    # the oracle on this rank's tokens, the full layer in the reference layout
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref_out, ref_idx, _ = orc.moe(H, E, K, I, Is, f(router).T.copy(), None,
                                  f(full.up_w).transpose(0, 2, 1).copy(), None,
                                  f(full.down_w).transpose(0, 2, 1).copy(), None,
                                  f(full.shared_up_w).T.copy(), None,
                                  f(full.shared_down_w).T.copy(), None, f(x), x.shape[0],
                                  orc.SIGMOID_RENORM)
    got = out.float().cpu().numpy().reshape(-1, H)
    rel = float(np.max(np.abs(got - ref_out.reshape(-1, H))) / np.max(np.abs(ref_out)))
    same_idx = bool(np.array_equal(idx.cpu().numpy(), ref_idx))
    q.put((rank, same_idx, rel, same_repeat))
    if mode != "nccl":
        ep.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["native", "native_pull", "peer", "peer2", "nccl"],
                         ids=["native_c_abi_push", "native_c_abi_pull", "nvlink_peer_stores",
                              "nvlink_peer_stores_2_phases", "nccl_all_to_all"])
def test_expert_parallel_two_gpus_matches_oracle(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same_idx, err, same_repeat in res:
        assert same_idx, rank
        assert err <= 2e-2, (rank, err)
        assert same_repeat, rank
