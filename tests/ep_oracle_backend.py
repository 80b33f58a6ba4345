"""A CPU compute backend for nk_ep.ExpertParallelMoe built on the oracle
(test infrastructure): the same stage contract as nk_ep.NkBackend, with the
reference arithmetic (oracle/nk_oracle.c) on float32 host tensors."""
import numpy as np
import torch

import oracle as orc


class OracleBackend:
    def __init__(self, H, E, K, I, Is, mode, router_kn, up_kn_local, down_kn_local, sup_kn,
                 sdown_kn):
        self.H, self.E, self.K, self.I, self.Is, self.mode = H, E, K, I, Is, mode
        self.router_kn, self.up, self.down = router_kn, up_kn_local, down_kn_local
        self.sup, self.sdown = sup_kn, sdown_kn

    def dispatch(self, x):
        xn = x.numpy()
        t = xn.shape[0]
        scores = orc.linear(self.router_kn, None, self.H, self.E, xn, t)
        idx, w = orc.route(scores, t, self.E, self.K, self.mode)
        counts, offs, perm = orc.route_histogram(idx, t, self.K, self.E)
        slot_pos = np.empty(t * self.K, np.int32)
        slot_pos[perm] = np.arange(t * self.K, dtype=np.int32)
        rows = xn[perm // self.K]
        return (torch.from_numpy(idx), torch.from_numpy(w), torch.from_numpy(counts),
                torch.from_numpy(slot_pos), torch.from_numpy(np.ascontiguousarray(rows)))

    def experts(self, rows, seg_expert, seg_rows):
        r = rows.numpy()
        out = np.zeros_like(r)
        off = 0
        for e, n in zip(seg_expert.tolist(), seg_rows.tolist()):
            if n:
                out[off:off + n] = orc.mlp(self.H, self.I, self.up[e], None, self.down[e], None,
                                           r[off:off + n], n).reshape(n, self.H)
            off += n
        return torch.from_numpy(out)

    def shared(self, x):
        if not self.Is:
            return None
        t = x.shape[0]
        return torch.from_numpy(orc.mlp(self.H, self.Is, self.sup, None, self.sdown, None,
                                        x.numpy(), t).reshape(t, self.H))

    def combine(self, y, sh, w, slot_pos, tokens, out_dtype):
        yn, wn, pos = y.numpy(), w.numpy(), slot_pos.numpy()
        out = np.zeros((tokens, self.H), np.float32)
        if sh is not None:
            out = out + sh.numpy()
        for r in range(self.K):
            sel = pos[np.arange(tokens) * self.K + r]
            out = out + wn[np.arange(tokens) * self.K + r][:, None] * yn[sel]
        return torch.from_numpy(out.astype(np.float32))
