"""Golden vectors of the reference predictor's optional score terms, run on
CPU in the build container:

    PYTHONPATH=<path to the reference checkout> python tests/golden/make_predictor_terms.py

For `inputs.PREDICTOR_TERMS`: a reference `LayerPredictor` with the count
term and a rank-r second-order head (seeded parameters) scores seeded
pooled features of a head subset; the file holds its logits, the logits
of the same projections without the terms, and the gradients of a seeded
linear functional of the logits with respect to so_q, so_k and count_gain.
It also holds the products so_q so_k^T that `init_low_rank_second_order_`
gives for seeded moments, at rank r and at full rank. Writes
`tests/golden/predictor_terms.npz`.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import inputs  # noqa: E402

from miowtion.veda import predictor as veda_predictor  # noqa: E402


def main() -> None:
    spec = inputs.PREDICTOR_TERMS
    heads, dim, rank = spec['heads'], spec['dim'], spec['rank']
    tensors = inputs.predictor_term_inputs(spec)
    sub = tensors['heads']
    full = veda_predictor.LayerPredictor(heads, dim, rank, count_term=True)
    plain = veda_predictor.LayerPredictor(heads, dim)
    with torch.no_grad():
        for name in ('proj_q', 'proj_k', 'so_q', 'so_k', 'count_gain'):
            getattr(full, name).copy_(tensors[name])
        plain.proj_q.copy_(tensors['proj_q'])
        plain.proj_k.copy_(tensors['proj_k'])
    logits = full(tensors['feats_q'], tensors['feats_k'], sub,
                  sq_q=tensors['sq_q'], var_k=tensors['var_k'],
                  log_count=tensors['log_count'])
    (logits * tensors['probe']).sum().backward()
    out = {'logits': logits.detach().numpy(),
           'plain': plain(tensors['feats_q'], tensors['feats_k'],
                          sub).detach().numpy(),
           'grad_so_q': full.so_q.grad.numpy(),
           'grad_so_k': full.so_k.grad.numpy(),
           'grad_count_gain': full.count_gain.grad.numpy()}
    c_u, c_v = inputs.predictor_term_moments(spec)
    for r in (rank, dim):
        layer = veda_predictor.LayerPredictor(c_u.shape[0], dim, r)
        layer.init_low_rank_second_order_(c_u, c_v)
        out[f'low_rank_{r}'] = torch.bmm(
            layer.so_q, layer.so_k.transpose(1, 2)).detach().numpy()
    path = os.path.join(HERE, 'predictor_terms.npz')
    np.savez_compressed(path, **out)
    print(f'wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)')


if __name__ == '__main__':
    main()
