"""Generate golden vectors for training-mode selective attention from the reference.

Runs nmquan1503/selective-attention's own ``SelectiveMHA`` (``modules/selective_attention.py``)
in training mode on CPU (fp32) and records the inputs and outputs of the part the CUDA
op replaces (``:232-280``: the score statistics, the std-scaled log-gates, the seq-mode gated
softmax and ``@ v``), with the gradients torch's autograd gives for them:

- ``q_rot, k_rot``: the outputs of the layer's ``rope`` (captured by wrapping it);
- ``v``: ``v_proj``'s output, as a leaf (forward hook), viewed as ``(b, H, L, D)``;
- ``select_gate``: ``sigmoid`` of ``gate_proj``'s output (a leaf through a forward hook),
  its gradient recovered from the leaf's as ``dz / (s (1 - s))``;
- ``out``: the attention output, from the layer's output with ``out_proj`` replaced by the
  identity (``hidden = out * out_gate``), and ``dout`` = the loss weights times ``out_gate``;
- ``std``: from ``score_std_ema`` after one step from zero (``0.1 std``).

Needs the reference checkout; run from the repository root:
``python tests/golden/make_golden_sattn_train.py``.
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_interp  # noqa: E402  (puts the reference on sys.path)

ref_interp.load()

import torch  # noqa: E402
import torch.nn as nn  # noqa: E402
from selective_attention.modules.selective_attention import SelectiveMHA  # noqa: E402


class _Capture(nn.Module):
    def __init__(self, rope, store):
        super().__init__()
        self.rope, self.store = rope, store

    def forward(self, q, k, positions, mode="seq"):
        q_rot, k_rot = self.rope(q, k, positions, mode=mode)
        q_rot.retain_grad()
        k_rot.retain_grad()
        self.store["q_rot"], self.store["k_rot"] = q_rot, k_rot
        return q_rot, k_rot


def run(seed, b, L, dim, head_dim, penalty, is_causal, lengths):
    torch.manual_seed(seed)
    H = dim // head_dim
    mha = SelectiveMHA(0, dim, head_dim, penalty, is_causal).train()
    with torch.no_grad():  # spread the gate bias (2.0 at init) so gates differ per head and token
        mha.gate_proj.bias.normal_(1.0, 1.0)
    store = {}
    mha.rope = _Capture(mha.rope, store)
    mha.out_proj = nn.Identity()

    def leaf_hook(name):
        def hook(module, inp, out):
            z = out.detach().requires_grad_(True)
            store[name] = z
            return z
        return hook

    mha.v_proj.register_forward_hook(leaf_hook("v_flat"))
    mha.gate_proj.register_forward_hook(leaf_hook("z"))
    x = torch.randn(b, L, dim)
    lens = None if lengths is None else torch.tensor(lengths, dtype=torch.long)
    hidden = mha(x, lens)
    R = torch.randn(b, L, dim)
    (hidden * R).sum().backward()

    z = store["z"]
    s = torch.sigmoid(z.detach())
    sel, og = s[..., :H], s[..., H:]
    to_bhld = lambda t: t.view(b, L, H, head_dim).transpose(1, 2).contiguous()  # noqa: E731
    out = to_bhld(hidden.detach() / og)
    dout = to_bhld(R * og)
    dsel = (z.grad[..., :H] / (sel * (1 - sel))).transpose(1, 2).contiguous()
    return {
        "q_rot": store["q_rot"].detach().clone(), "k_rot": store["k_rot"].detach().clone(),
        "v": to_bhld(store["v_flat"].detach()), "select_gate": sel.transpose(1, 2).contiguous(),
        "lengths": lens, "log_gate_penalty": penalty, "is_causal": is_causal, "scale": head_dim ** -0.5,
        "dout": dout, "out": out, "std": (mha.score_std_ema / 0.1).clone(),
        "q_rot_grad": store["q_rot"].grad.clone(), "k_rot_grad": store["k_rot"].grad.clone(),
        "v_grad": to_bhld(store["v_flat"].grad), "select_gate_grad": dsel,
    }


CASES = {
    # causal LM block, ragged rows (lengths), L not a multiple of the 64-token tile
    "sattn_train_causal_ragged_fp32": dict(seed=1, b=2, L=80, dim=64, head_dim=16, penalty=1.0, is_causal=True,
                                           lengths=[80, 53]),
    # bidirectional block (bi_block.py: is_causal=False) with padding
    "sattn_train_bidir_ragged_fp32": dict(seed=2, b=3, L=70, dim=64, head_dim=32, penalty=0.5, is_causal=False,
                                          lengths=[70, 41, 9]),
    # causal, no lengths, head_dim 64, two key tiles
    "sattn_train_causal_d64_fp32": dict(seed=3, b=1, L=130, dim=128, head_dim=64, penalty=2.0, is_causal=True,
                                        lengths=None),
}

if __name__ == "__main__":
    for name, kw in CASES.items():
        torch.save(run(**kw), os.path.join(HERE, name + ".pt"))
        print("wrote", name)
