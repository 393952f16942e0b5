"""Golden vectors for one Qwen3.5 Gated DeltaNet decode step (after the input
projections), made with the installed transformers package's own functions
(transformers/models/qwen3_5/modeling_qwen3_5.py): torch_causal_conv1d_update,
torch_recurrent_gated_delta_rule (with its l2norm of q and k) and
Qwen3_5RMSNormGated, wired as Qwen3_5GatedDeltaNet.forward wires them for one
cached token.  Seeded inputs, 2 key heads / 4 value heads of 128 (the 9B has
16 / 32), three consecutive steps from a random state.

The fixture stores the states in this repository's layout: the conv history
as a 4-slot circular buffer (input of position p in slot p % 4) and the
recurrent state as S[h][j][i] (value j, key i; transformers keeps [h][i][j]).

    python tests/golden/gen_deltanet.py     # writes tests/golden/deltanet_step.npz
"""
import os

import numpy as np
import torch
import torch.nn.functional as F
from transformers.models.qwen3_5 import modeling_qwen3_5 as M

HERE = os.path.dirname(os.path.abspath(__file__))
NK, NV, DK, DV, KS, STEPS, T0, EPS = 2, 4, 128, 128, 4, 3, 5, 1e-6


def main():
    g = torch.Generator().manual_seed(1234)
    conv_dim = 2 * NK * DK + NV * DV
    rnd = lambda *s, scale=1.0: (torch.randn(*s, generator=g) * scale).float()
    conv_w = rnd(conv_dim, KS, scale=0.5)
    a_log = torch.log(torch.rand(NV, generator=g) * 15.0 + 1.0)
    dt_bias = rnd(NV, scale=0.5)
    norm_w = 1.0 + rnd(DV, scale=0.1)
    # transformers' cache: the last KS inputs, oldest first
    conv_state = rnd(1, conv_dim, KS)
    rec_state = rnd(1, NV, DK, DV, scale=0.05)
    norm = M.Qwen3_5RMSNormGated(DV, eps=EPS)
    norm.weight.data.copy_(norm_w)

    # this repository's layout of the initial states (position of the first step: T0)
    hist = np.zeros((4, conv_dim), np.float32)
    for back in (1, 2, 3, 4):  # input of position T0 - back = conv_state[..., KS - back]
        hist[(T0 - back) % 4] = conv_state[0, :, KS - back].numpy()
    state0 = rec_state[0].transpose(1, 2).contiguous().numpy()  # [h][j][i]

    ins = {k: [] for k in ("mixed", "z", "a", "b")}
    outs = []
    for _ in range(STEPS):
        mixed = rnd(1, conv_dim, 1)
        z = rnd(1, 1, NV, DV)
        a = rnd(1, 1, NV)
        b = rnd(1, 1, NV)
        u = M.torch_causal_conv1d_update(mixed, conv_state, conv_w, None, "silu")  # updates conv_state
        u = u.transpose(1, 2)
        q, k, v = torch.split(u, [NK * DK, NK * DK, NV * DV], dim=-1)
        q = q.reshape(1, 1, NK, DK).repeat_interleave(NV // NK, dim=2)
        k = k.reshape(1, 1, NK, DK).repeat_interleave(NV // NK, dim=2)
        v = v.reshape(1, 1, NV, DV)
        beta = b.sigmoid()
        gg = -a_log.float().exp() * F.softplus(a.float() + dt_bias)
        o, rec_state = M.torch_recurrent_gated_delta_rule(q, k, v, g=gg, beta=beta, initial_state=rec_state,
                                                         output_final_state=True, use_qk_l2norm_in_kernel=True)
        o = norm(o.reshape(-1, DV), z.reshape(-1, DV)).reshape(-1)
        ins["mixed"].append(mixed.reshape(-1).numpy())
        ins["z"].append(z.reshape(-1).numpy())
        ins["a"].append(a.reshape(-1).numpy())
        ins["b"].append(b.reshape(-1).numpy())
        outs.append(o.detach().numpy())
    hist_end = np.zeros((4, conv_dim), np.float32)
    for back in (1, 2, 3, 4):
        hist_end[(T0 + STEPS - back) % 4] = conv_state[0, :, KS - back].numpy()
    np.savez_compressed(
        os.path.join(HERE, "deltanet_step.npz"),
        nk=NK, nv=NV, dk=DK, dv=DV, t0=T0, eps=EPS,
        conv_w=conv_w.numpy(), a_log=a_log.numpy(), dt_bias=dt_bias.numpy(), norm_w=norm_w.numpy(),
        hist0=hist, state0=state0,
        mixed=np.stack(ins["mixed"]), z=np.stack(ins["z"]), a=np.stack(ins["a"]), b=np.stack(ins["b"]),
        out=np.stack(outs), hist_end=hist_end,
        state_end=rec_state[0].transpose(1, 2).contiguous().numpy(),
    )


if __name__ == "__main__":
    main()
