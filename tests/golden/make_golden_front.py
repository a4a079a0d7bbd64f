"""Golden vectors for the SSM prefill front end, made by the reference's own code.

Builds the reference ``SSM`` module on CPU (``modules/ssm.py``) and runs the statements
of its ``forward`` between the input projection and the scan (``:112-134``) with the
module's own depthwise ``conv`` layer, plus ``SSMCache.build_conv_ctx``
(``inference/ssm_cache.py``), on seeded inputs; saves inputs and outputs as
``ssm_front_<case>.pt``. Needs the reference checkout; run from the repository root:
``python tests/golden/make_golden_front.py``.
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_interp  # noqa: E402  (sets TRITON_INTERPRET before triton loads)

ref_interp.load()

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402
from selective_attention.inference import SSMCache  # noqa: E402
from selective_attention.modules.ssm import SSM  # noqa: E402


def case(name, seed, b, L, model_dim, state_dim, head_dim, groups, K, lengths, dtype):
    torch.manual_seed(seed)
    ssm = SSM(layer_idx=0, model_dim=model_dim, state_dim=state_dim, conv_kernel_size=K, head_dim=head_dim,
              num_groups=groups, device="cpu").to(dtype)
    inner, gn = ssm.inner_dim, ssm.num_groups * ssm.state_dim
    g = torch.Generator().manual_seed(seed + 1)
    hBC = torch.randn(b, L, inner + 2 * gn, generator=g).to(dtype)
    with torch.no_grad():
        hBC_t = hBC.transpose(1, 2)                       # modules/ssm.py:119
        cache = SSMCache()
        cache.build_conv_ctx(hBC_t, lengths, K)           # :121-123
        s = F.silu(hBC_t)                                 # :125
        out = ssm.conv(s).transpose(1, 2)[:, :L]          # :126-127
        x, B, C = torch.split(out, [inner, gn, gn], dim=-1)  # :129-134
    torch.save({"hBC": hBC, "weight": ssm.conv.weight.detach().clone(), "bias": ssm.conv.bias.detach().clone(),
                "inner": inner, "gn": gn, "K": K, "lengths": lengths, "x": x.contiguous(), "B": B.contiguous(),
                "C": C.contiguous(), "conv_ctx": cache.conv_ctx.contiguous()},
               os.path.join(HERE, f"ssm_front_{name}.pt"))
    print(name, tuple(hBC.shape), dtype)


def decode_case(name, seed, b, model_dim, state_dim, head_dim, groups, K, dtype, steps=2):
    """Two decode steps of the reference's own code (modules/ssm.py:173-186 with
    SSMCache.update): inputs hBC per step and the starting cache, outputs per step."""
    torch.manual_seed(seed)
    ssm = SSM(layer_idx=0, model_dim=model_dim, state_dim=state_dim, conv_kernel_size=K, head_dim=head_dim,
              num_groups=groups, device="cpu").to(dtype)
    inner, gn = ssm.inner_dim, ssm.num_groups * ssm.state_dim
    g = torch.Generator().manual_seed(seed + 1)
    cache = SSMCache()
    cache.conv_ctx = torch.randn(b, inner + 2 * gn, K, generator=g).to(dtype)
    ctx0 = cache.conv_ctx.clone()
    hs, outs = [], []
    with torch.no_grad():
        for _ in range(steps):
            hBC = torch.randn(b, inner + 2 * gn, generator=g).to(dtype)
            cache.update(hBC)                                                      # :173
            h = F.silu(cache.conv_ctx)                                             # :174-175
            h = (h * ssm.conv.weight.squeeze(1)).sum(dim=-1) + ssm.conv.bias       # :176
            x, B, C = torch.split(h, [inner, gn, gn], dim=-1)                     # :177-184
            hs.append(hBC)
            outs.append({"x": x.contiguous(), "B": B.contiguous(), "C": C.contiguous(),
                         "conv_ctx": cache.conv_ctx.clone()})
    torch.save({"ctx0": ctx0, "hBC": hs, "out": outs, "weight": ssm.conv.weight.detach().clone(),
                "bias": ssm.conv.bias.detach().clone(), "inner": inner, "gn": gn, "K": K},
               os.path.join(HERE, f"ssm_decode_{name}.pt"))
    print(name, b, inner + 2 * gn, dtype)


if __name__ == "__main__":
    decode_case("fp32", 8, 3, 64, 16, 16, 2, 4, torch.float32)
    decode_case("bf16", 9, 4, 128, 32, 32, 1, 4, torch.bfloat16)
    case("fp32", 5, 3, 70, 64, 16, 16, 2, 4, torch.tensor([70, 33, 2]), torch.float32)
    case("fp32_short", 6, 2, 3, 32, 8, 16, 1, 4, None, torch.float32)
    case("bf16", 7, 2, 130, 128, 32, 32, 1, 4, torch.tensor([130, 97]), torch.bfloat16)
