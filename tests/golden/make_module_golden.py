"""Generate tests/golden/modules/*.npz from the reference's own nn.Modules.

Run in a container where the reference package source is available:

    MSDA_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_module_golden.py

It builds the reference's MSDA2D / MSDA3D modules
(src/msda_triton/pytorch/msda_2d.py:117-383, src/msda_triton/pytorch/msda_3d.py:121-394,
which sample with grid_sample), runs init_weights() from a fixed torch seed
(stored as init/<param>), perturbs every parameter with seeded noise (so the
offsets and weights are not the init pattern; stored as param/<param>), runs
forward and backward in float32 on the CPU and stores the inputs, the output
and the gradients of the inputs and parameters.  The GPU box does not have
the reference; the tests only read the stored files.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "modules")

# name: ndim, module kwargs, bs, nq, shapes, options
CASES = {
    "mod3d_default": (3, dict(embed_dims=64, num_heads=4, num_levels=2, num_points=3, dropout=0.0),
                      2, 40, [(4, 6, 6), (2, 3, 3)], dict(query_pos=True, mask=True)),
    "mod3d_batch_first_chunked": (3, dict(embed_dims=32, num_heads=2, num_levels=3, num_points=2,
                                          dropout=0.0, batch_first=True, query_chunk_size=7,
                                          head_chunk_size=1, use_checkpoint=True),
                                  1, 20, [(6, 8, 8), (3, 4, 4), (2, 2, 2)], dict(train=True)),
    "mod3d_self_attention": (3, dict(embed_dims=32, num_heads=4, num_levels=2, num_points=2,
                                     dropout=0.0, clamp_grid=False),
                             2, None, [(3, 4, 5), (2, 2, 3)], dict(value_none=True, identity=True)),
    "mod2d_default": (2, dict(embed_dims=64, num_heads=8, num_levels=3, num_points=4, dropout=0.0),
                      2, 30, [(12, 16), (6, 8), (3, 4)], dict(query_pos=True, mask=True)),
    "mod2d_batch_first_chunked": (2, dict(embed_dims=48, num_heads=6, num_levels=2, num_points=3,
                                          dropout=0.0, batch_first=True, query_chunk_size=11,
                                          head_chunk_size=4, use_checkpoint=True, clamp_eps=0.05),
                                  2, 25, [(10, 12), (5, 6)], dict(train=True)),
}


def _reference():
    src = os.environ.get("MSDA_REFERENCE_SRC")
    if not src:
        raise SystemExit("set MSDA_REFERENCE_SRC to the reference's src/ directory")
    sys.path.insert(0, src)
    from msda_triton.pytorch.msda_2d import MSDA2D
    from msda_triton.pytorch.msda_3d import MSDA3D

    return {2: MSDA2D, 3: MSDA3D}


def make_case(cls, ndim, kw, bs, nq, shapes, opt, seed):
    torch.manual_seed(seed)
    m = cls(**kw)
    m.init_weights()
    init = {k: v.detach().clone() for k, v in m.state_dict().items()}
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.05 * torch.randn(p.shape, generator=g))
    m.train(bool(opt.get("train")))
    E = kw["embed_dims"]
    K = int(sum(int(np.prod(s)) for s in shapes))
    nq = K if opt.get("value_none") else nq
    bf = kw.get("batch_first", False)
    shape_q = (bs, nq, E) if bf else (nq, bs, E)
    shape_v = (bs, K, E) if bf else (K, bs, E)
    query = torch.randn(shape_q, generator=g)
    value = torch.randn(shape_v, generator=g)
    query_pos = torch.randn(shape_q, generator=g) if opt.get("query_pos") else None
    identity = torch.randn(shape_q, generator=g) if opt.get("identity") else None
    ref = torch.rand(bs, nq, len(shapes), ndim, generator=g) * 0.8 + 0.1
    mask = (torch.rand(bs, K, generator=g) < 0.1) if opt.get("mask") else None
    spatial = torch.tensor(shapes, dtype=torch.int64)
    query.requires_grad_(True)
    ref.requires_grad_(True)
    if not opt.get("value_none"):
        value.requires_grad_(True)
    out = m(query, value=None if opt.get("value_none") else value, identity=identity,
            query_pos=query_pos, key_padding_mask=mask, reference_points=ref,
            spatial_shapes=spatial)
    G = torch.randn(out.shape, generator=g)
    (out * G).sum().backward()
    rec = {"ndim": np.array(ndim), "shapes": spatial.numpy(), "query": query.detach().numpy(),
           "reference_points": ref.detach().numpy(), "out": out.detach().numpy(),
           "grad_out": G.numpy(), "grad_query": query.grad.numpy(),
           "grad_reference_points": ref.grad.numpy()}
    if not opt.get("value_none"):
        rec["value"] = value.detach().numpy()
        rec["grad_value"] = value.grad.numpy()
    for name, t in (("query_pos", query_pos), ("identity", identity), ("key_padding_mask", mask)):
        if t is not None:
            rec[name] = t.numpy()
    for k, v in init.items():
        rec["init/" + k] = v.numpy()
    for k, v in m.state_dict().items():
        rec["param/" + k] = v.numpy()
    for k, p in m.named_parameters():
        rec["grad/" + k] = p.grad.numpy()
    return rec


def main() -> None:
    classes = _reference()
    os.makedirs(OUT, exist_ok=True)
    for i, (name, (ndim, kw, bs, nq, shapes, opt)) in enumerate(CASES.items()):
        rec = make_case(classes[ndim], ndim, kw, bs, nq, shapes, opt, seed=100 + i)
        rec["init_seed"] = np.array(100 + i)
        rec["module_kwargs"] = np.array(repr(kw))
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **rec)
        print(name, {k: v.shape for k, v in rec.items() if not k.startswith(("init/", "param/", "grad/"))})


if __name__ == "__main__":
    main()
