"""Tile-score predictor: which key tiles each query tile should attend.

Mirror of the reference's `miowtion/veda/predictor.py` for the default
predictor: per tile, q and k are pooled into [mean | max | min]; per layer
and head a residual projection maps them to D dims,
    q_hat = pool_q @ P_q[h] + mean_q,   k_hat likewise,
and block logits are q_hat . k_hat / sqrt(D) in fp32. Pooling and logits run
in CUDA kernels (csrc/permute.cu, csrc/predict.cu).

The reference's optional terms (`count_term`, `second_order_rank > 0`) are
not implemented on the device and raise NotImplementedError.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from miowtion_b200 import _lib
from miowtion_b200 import tiling

INIT_STD = 1e-4  # predictor.py:70
SECOND_RAW = 'raw'
SECOND_CENTRAL = 'central'


@torch.no_grad()
def pool_tiles(x: torch.Tensor, layout: tiling.TileLayout,
               second: str | None = None) -> torch.Tensor:
    """Masked mean/max/min over the real rows of every tile
    (predictor.py:82-130): [N, H', D] bf16 -> [H', n, 3D] fp32, or the
    second moment [H', n, D] ('raw' E[x^2], 'central' Var(x))."""
    if second not in (None, SECOND_RAW, SECOND_CENTRAL):
        raise ValueError(f'unknown second moment {second!r}')
    tiling._check_rows(x, 'x')  # pylint: disable=protected-access
    if x.shape[0] != layout.num_slots:
        raise ValueError('x must be tile-ordered [num_slots, H\', D]')
    heads, dim = x.shape[1], x.shape[2]
    out = torch.empty(heads, layout.n_tiles, dim if second else 3 * dim,
                      dtype=torch.float32, device=x.device)
    feats = out if second is None else None
    sq = out if second == SECOND_RAW else None
    var = out if second == SECOND_CENTRAL else None
    _lib.call('veda_gather_pool', x.data_ptr(), x.stride(0), x.stride(1),
              None, layout.valid_count.data_ptr(), layout.n_tiles, None,
              heads, None, 0, 0, _lib.ptr(feats), _lib.ptr(sq),
              _lib.ptr(var), _lib.stream_ptr(x.device))
    return out


def _logits_and_embeddings(feats_q: torch.Tensor, feats_k: torch.Tensor,
                           proj_q: torch.Tensor, proj_k: torch.Tensor,
                           heads: torch.Tensor):
    """The kernel call: logits [H', n_q, n_k] and the tile embeddings q_hat
    [H', n_q, D], k_hat [H', n_k, D] it leaves in its workspace."""
    n_heads, n_q = feats_q.shape[0], feats_q.shape[1]
    n_k = feats_k.shape[1]
    lib = _lib.load()
    ws_bytes = lib.veda_predict_workspace(n_heads, n_q, n_k)
    workspace = torch.empty(n_heads * (n_q + n_k) * 128, dtype=torch.float32,
                            device=feats_q.device)
    if workspace.numel() * 4 < ws_bytes:
        raise RuntimeError('predictor workspace layout changed')
    logits = torch.empty(n_heads, n_q, n_k, dtype=torch.float32,
                         device=feats_q.device)
    _lib.call('veda_predict_logits', feats_q.data_ptr(), feats_k.data_ptr(),
              proj_q.data_ptr(), proj_k.data_ptr(), heads.data_ptr(),
              n_heads, n_q, n_k, logits.data_ptr(), workspace.data_ptr(),
              workspace.numel() * 4, _lib.stream_ptr(feats_q.device))
    q_hat = workspace[:n_heads * n_q * 128].view(n_heads, n_q, 128)
    k_hat = workspace[n_heads * n_q * 128:].view(n_heads, n_k, 128)
    return logits, q_hat, k_hat


class _PredictLogits(torch.autograd.Function):
    """Logits with gradients for the projections (the stage-1 teacher
    trains them, veda/attention.py:446-450). Forward: the fp32 kernel.
    Backward, with G = dL/dlogits / sqrt(D) and the features constant:
        dq_hat = G k_hat,  dk_hat = G^T q_hat,
        dP_q[heads[h]] += feats_q[h]^T dq_hat[h]  (and likewise for k)
    as fp32 batched GEMMs (the `mean` residual carries no parameter)."""

    @staticmethod
    def forward(ctx, feats_q, feats_k, proj_q, proj_k, heads):
        logits, q_hat, k_hat = _logits_and_embeddings(
            feats_q, feats_k, proj_q.detach(), proj_k.detach(), heads)
        ctx.save_for_backward(feats_q, feats_k, q_hat, k_hat, heads)
        ctx.proj_shapes = (proj_q.shape, proj_k.shape)
        return logits

    @staticmethod
    def backward(ctx, grad):
        feats_q, feats_k, q_hat, k_hat, heads = ctx.saved_tensors
        g = grad.float() / math.sqrt(q_hat.shape[-1])
        d_qhat = torch.bmm(g, k_hat)
        d_khat = torch.bmm(g.transpose(1, 2), q_hat)
        grads = []
        for feats, d_hat, shape in ((feats_q, d_qhat, ctx.proj_shapes[0]),
                                    (feats_k, d_khat, ctx.proj_shapes[1])):
            per_head = torch.bmm(feats.transpose(1, 2), d_hat)
            grads.append(torch.zeros(shape, dtype=torch.float32,
                                     device=feats.device).index_add_(
                                         0, heads, per_head))
        return None, None, grads[0], grads[1], None


def predict_logits(feats_q: torch.Tensor, feats_k: torch.Tensor,
                   proj_q: torch.Tensor, proj_k: torch.Tensor,
                   heads: torch.Tensor) -> torch.Tensor:
    """[H', n_q, n_k] fp32 logits of pooled features (predictor.py:251-338);
    differentiable in proj_q / proj_k when they require gradients."""
    if feats_q.dim() != 3 or feats_q.shape[-1] != 3 * 128:
        raise ValueError('features must be [H\', n, 384]')
    if not feats_q.is_cuda:
        raise RuntimeError('the predictor kernels run on CUDA only')
    heads = heads.to(device=feats_q.device, dtype=torch.int64).contiguous()
    feats_q = feats_q.detach().float().contiguous()
    feats_k = feats_k.detach().float().contiguous()
    n_heads = feats_q.shape[0]
    if heads.numel() != n_heads or feats_k.shape[0] != n_heads:
        raise ValueError('heads and features disagree on the head count')
    if torch.is_grad_enabled() and (proj_q.requires_grad
                                    or proj_k.requires_grad):
        if proj_q.dtype != torch.float32 or proj_k.dtype != torch.float32:
            raise NotImplementedError('trainable projections must be fp32')
        return _PredictLogits.apply(feats_q, feats_k, proj_q.contiguous(),
                                    proj_k.contiguous(), heads)
    return _logits_and_embeddings(feats_q, feats_k,
                                  proj_q.detach().float().contiguous(),
                                  proj_k.detach().float().contiguous(),
                                  heads)[0]


class LayerPredictor(nn.Module):
    """Projections of one layer: proj_q, proj_k [num_heads, 3D, D]
    (predictor.py:197-230)."""

    def __init__(self, num_heads: int, head_dim: int,
                 second_order_rank: int = 0, count_term: bool = False):
        super().__init__()
        if second_order_rank or count_term:
            raise NotImplementedError(
                'second-order and count terms have no B200 kernel')
        self.head_dim = head_dim
        self.second_order_rank = 0
        self.proj_q = nn.Parameter(torch.empty(num_heads, 3 * head_dim,
                                               head_dim))
        self.proj_k = nn.Parameter(torch.empty(num_heads, 3 * head_dim,
                                               head_dim))
        nn.init.normal_(self.proj_q, std=INIT_STD)
        nn.init.normal_(self.proj_k, std=INIT_STD)

    def forward(self, feats_q: torch.Tensor, feats_k: torch.Tensor,
                heads: torch.Tensor) -> torch.Tensor:
        """Block logits [H', n_q, n_k] fp32 (predictor.py:299-338).

        Raises:
            NotImplementedError: For a head_dim other than 128 (the scoring
                kernel's only size; other sizes load and save, nothing more).
        """
        if self.head_dim != 128:
            raise NotImplementedError('the predictor kernels take head_dim 128')
        return predict_logits(feats_q, feats_k, self.proj_q, self.proj_k,
                              heads)


class TileScorePredictor(nn.Module):
    """All layers: `layers.{i}.proj_q` / `layers.{i}.proj_k`
    (predictor.py:341-410). Kept replicated across devices."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int,
                 second_order_rank: int = 0, count_term: bool = False):
        super().__init__()
        self.second_order_rank = second_order_rank
        self.count_term = count_term
        self.layers = nn.ModuleList(
            LayerPredictor(num_heads, head_dim, second_order_rank, count_term)
            for _ in range(num_layers))

    def scores(self, layer: int, q_tiles: torch.Tensor, k_tiles: torch.Tensor,
               layout: tiling.TileLayout, heads: torch.Tensor) -> torch.Tensor:
        """Block logits of one head group [H', n, n] fp32."""
        feats_q = pool_tiles(q_tiles, layout)
        feats_k = pool_tiles(k_tiles, layout)
        return self.layers[layer](feats_q, feats_k, heads)
