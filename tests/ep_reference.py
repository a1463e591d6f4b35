"""CPU stand-ins for the per-rank EP kernels (test infrastructure): they
restate ep_pack / ep_unpack / the local expert compute in numpy with the CPU
oracle so the exchange logic of nki_moe_7013_b200.ep can run under gloo."""
import numpy as np
import torch

from oracle import oracle


def pack_np(idx: np.ndarray, tw: np.ndarray, x: torch.Tensor, e_local: int, n_ranks: int):
    T, k = idx.shape
    dest = idx // e_local
    order = sorted(range(T * k), key=lambda p: (dest.reshape(-1)[p], p))  # stable by (token, slot)
    counts = np.bincount(dest.reshape(-1), minlength=n_ranks).astype(np.int32)
    pair_pos = np.empty(T * k, np.int32)
    for r, p in enumerate(order):
        pair_pos[p] = r
    rows = np.array([p // k for p in order], dtype=np.int64)
    send_expert = np.array([idx.reshape(-1)[p] - dest.reshape(-1)[p] * e_local for p in order], np.int32)
    send_w = np.array([tw.reshape(-1)[p] for p in order], np.float32)
    return dict(send_counts=counts, send_x=x[torch.from_numpy(rows)], send_expert=send_expert,
                send_w=send_w, pair_pos=pair_pos.reshape(T, k))


class CpuEPKernels:
    def router(self, x, w_router, k, normalize, bias):
        _, idx, tw = oracle.router(x, w_router, k, normalize)
        return torch.from_numpy(idx), torch.from_numpy(tw)

    def pack(self, idx, tw, x, e_local, n_ranks):
        p = pack_np(idx.numpy(), tw.numpy(), x, e_local, n_ranks)
        return dict(send_counts=torch.from_numpy(p["send_counts"]), send_x=p["send_x"],
                    send_expert=torch.from_numpy(p["send_expert"]), send_w=torch.from_numpy(p["send_w"]),
                    pair_pos=torch.from_numpy(p["pair_pos"]))

    def local_moe(self, recv_x, recv_expert, recv_w, local):
        H = recv_x.shape[1]
        if recv_x.shape[0] == 0:
            return torch.empty((0, H), dtype=torch.bfloat16)
        x = oracle.bf16_bits_to_f32(oracle.as_bf16_bits(recv_x))
        wgu = oracle.bf16_bits_to_f32(oracle.as_bf16_bits(local.gate_up))
        wd = oracle.bf16_bits_to_f32(oracle.as_bf16_bits(local.down))
        y = np.zeros((x.shape[0], H), np.float64)
        for r in range(x.shape[0]):
            e = int(recv_expert[r])
            a = oracle.expert_gate_up_swiglu(x[r:r + 1], wgu[e])
            y[r] = float(recv_w[r]) * (a.astype(np.float64) @ wd[e].astype(np.float64).T)[0]
        return torch.from_numpy(oracle.round_to_bf16(y.astype(np.float32))).to(torch.bfloat16)

    def unpack(self, y_back, pair_pos, residual):
        yb = y_back.float().numpy().astype(np.float64)
        pp = pair_pos.numpy()
        out = yb[pp].sum(axis=1)
        if residual is not None:
            out = out + residual.float().numpy()
        return torch.from_numpy(oracle.round_to_bf16(out.astype(np.float32))).to(torch.bfloat16)
