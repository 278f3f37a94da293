"""Tile-score predictor: which key tiles each query tile should attend.

Mirror of the reference's `miowtion/veda/predictor.py` for the default
predictor: per tile, q and k are pooled into [mean | max | min]; per layer
and head a residual projection maps them to D dims,
    q_hat = pool_q @ P_q[h] + mean_q,   k_hat likewise,
and block logits are q_hat . k_hat / sqrt(D) in fp32. Pooling and logits run
in CUDA kernels (csrc/permute.cu, csrc/predict.cu).

The reference's optional score terms are supported on top of that kernel:
`count_term` adds a learned per-head gain times log B_j (B_j = the real
rows of key tile j), and `second_order_rank = r > 0` a low-rank
second-cumulant head (sq_q @ So_q) . (var_k @ So_k) over the pooled E[q^2]
and Var(k), which the gather/pool kernel produces in the same pass. Both
are small fp32 batched products next to the logits (r / D of the logit
GEMM's work), with autograd for their parameters.
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


def _psd_roots(matrix: torch.Tensor,
               floor: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric square root of a PSD matrix and the pseudo-inverse of that
    root, dropping eigenvalues at or below `floor` times the largest
    (predictor.py:171-194)."""
    values, vectors = torch.linalg.eigh(matrix)
    values = values.clamp(min=0.0)
    cut = float(values.max()) * floor
    kept = values > cut
    root = torch.where(kept, values.sqrt(), 0.0)
    inverse = torch.where(kept, values.clamp(min=cut).rsqrt(), 0.0)
    basis_t = vectors.transpose(0, 1)
    return (vectors * root) @ basis_t, (vectors * inverse) @ basis_t


class LayerPredictor(nn.Module):
    """Projections of one layer: proj_q, proj_k [num_heads, 3D, D]
    (predictor.py:197-230); with `second_order_rank = r` also so_q, so_k
    [num_heads, D, r], with `count_term` a gain [num_heads] on log B_j
    (initialised to 1, the exact coefficient)."""

    def __init__(self, num_heads: int, head_dim: int,
                 second_order_rank: int = 0, count_term: bool = False):
        super().__init__()
        if not 0 <= second_order_rank <= head_dim:
            raise ValueError(f'second_order_rank {second_order_rank} must be '
                             f'in [0, {head_dim}]')
        self.head_dim = head_dim
        self.second_order_rank = second_order_rank
        self.proj_q = nn.Parameter(torch.empty(num_heads, 3 * head_dim,
                                               head_dim))
        self.proj_k = nn.Parameter(torch.empty(num_heads, 3 * head_dim,
                                               head_dim))
        nn.init.normal_(self.proj_q, std=INIT_STD)
        nn.init.normal_(self.proj_k, std=INIT_STD)
        if second_order_rank:
            self.so_q = nn.Parameter(torch.empty(num_heads, head_dim,
                                                 second_order_rank))
            self.so_k = nn.Parameter(torch.empty(num_heads, head_dim,
                                                 second_order_rank))
            nn.init.normal_(self.so_q, std=INIT_STD)
            nn.init.normal_(self.so_k, std=INIT_STD)
        if count_term:
            self.count_gain = nn.Parameter(torch.ones(num_heads))

    @torch.no_grad()
    def init_exact_second_order_(self) -> None:
        """Sets the full-rank head to the diagonal cumulant term
        E[q^2] . Var(k) / (2 D): both sides sqrt(1 / (2 D)) times the
        identity (predictor.py:232-249).

        Raises:
            ValueError: If the rank is not head_dim.
        """
        if self.second_order_rank != self.head_dim:
            raise ValueError('the exact term needs second_order_rank == '
                             f'head_dim, not {self.second_order_rank}')
        scaled = torch.eye(self.head_dim, dtype=self.so_q.dtype,
                           device=self.so_q.device) * math.sqrt(
                               0.5 / self.head_dim)
        self.so_q.copy_(scaled)
        self.so_k.copy_(scaled)

    @torch.no_grad()
    def init_low_rank_second_order_(self, c_u: torch.Tensor,
                                    c_v: torch.Tensor,
                                    floor: float = 1e-6) -> None:
        """The rank-r head closest to (1 / 2D) I under the feature moments
        C_u = E[sq_q^T sq_q], C_v = E[var_k^T var_k] [num_heads, D, D]
        (predictor.py:258-297): per head the rank-r truncated SVD
        L S R^T of (1 / 2D) C_u^(1/2) C_v^(1/2), mapped back to each side,
        so_q = C_u^(-1/2) L_r S_r^(1/2), so_k = C_v^(-1/2) R_r S_r^(1/2).
        At r = D it reproduces `init_exact_second_order_`'s product on the
        moments' support.

        Raises:
            ValueError: Without a second-order head, or on moments of the
                wrong shape.
        """
        if not self.second_order_rank:
            raise ValueError('no second-order head to initialize')
        heads, dim = self.so_q.shape[0], self.head_dim
        for name, moment in (('c_u', c_u), ('c_v', c_v)):
            if tuple(moment.shape) != (heads, dim, dim):
                raise ValueError(f'{name} has shape {tuple(moment.shape)}, '
                                 f'expected {(heads, dim, dim)}')
        rank = self.second_order_rank
        for head in range(heads):
            root_u, inv_u = _psd_roots(c_u[head].float(), floor)
            root_v, inv_v = _psd_roots(c_v[head].float(), floor)
            left, sing, right_t = torch.linalg.svd(
                (0.5 / dim) * (root_u @ root_v))
            gain = sing[:rank].clamp(min=0.0).sqrt()
            self.so_q[head] = (inv_u @ left[:, :rank]) * gain
            self.so_k[head] = (inv_v @ right_t[:rank].transpose(0, 1)) * gain

    def _check_terms(self, sq_q, var_k, log_count) -> None:
        if hasattr(self, 'count_gain') != (log_count is not None):
            raise ValueError('log_count and count_term must be set '
                             'together')
        if bool(self.second_order_rank) != (sq_q is not None
                                            and var_k is not None):
            raise ValueError('second-order features and second_order_rank '
                             'must be set together')

    def optional_terms(self, heads: torch.Tensor,
                       sq_q: torch.Tensor | None = None,
                       var_k: torch.Tensor | None = None,
                       log_count: torch.Tensor | None = None
                       ) -> torch.Tensor | None:
        """The count and second-order terms [H', n_q, n_k] fp32 that
        `forward` adds to the bilinear logits (predictor.py:331-338), or
        None for a plain predictor. Differentiable in count_gain, so_q and
        so_k."""
        self._check_terms(sq_q, var_k, log_count)
        heads = heads.to(dtype=torch.int64)
        terms = None
        if log_count is not None:
            gain = self.count_gain.index_select(0, heads).float()
            terms = gain[:, None, None] * log_count.float()[None, None, :]
        if self.second_order_rank:
            u = torch.bmm(sq_q.float(),
                          self.so_q.index_select(0, heads).float())
            w = torch.bmm(var_k.float(),
                          self.so_k.index_select(0, heads).float())
            second = torch.bmm(u, w.transpose(1, 2))
            terms = second if terms is None else terms + second
        return terms

    def forward(self, feats_q: torch.Tensor, feats_k: torch.Tensor,
                heads: torch.Tensor, sq_q: torch.Tensor | None = None,
                var_k: torch.Tensor | None = None,
                log_count: torch.Tensor | None = None) -> torch.Tensor:
        """Block logits [H', n_q, n_k] fp32 (predictor.py:299-338).

        Args:
            feats_q, feats_k: [H', n, 3D] pooled features.
            heads: [H'] global head indices.
            sq_q: [H', n_q, D] pooled E[q^2]; iff second_order_rank > 0.
            var_k: [H', n_k, D] pooled Var(k); likewise.
            log_count: [n_k] log of each key tile's real rows (clamped to
                >= 1); iff count_term.

        Raises:
            ValueError: If an optional feature is missing, or given when
                its term is off.
            NotImplementedError: For a head_dim other than 128 (the scoring
                kernel's only size; other sizes load and save, nothing more).
        """
        self._check_terms(sq_q, var_k, log_count)
        if self.head_dim != 128:
            raise NotImplementedError('the predictor kernels take head_dim 128')
        logits = predict_logits(feats_q, feats_k, self.proj_q, self.proj_k,
                                heads)
        terms = self.optional_terms(heads.to(feats_q.device), sq_q, var_k,
                                    log_count)
        return logits if terms is None else logits + terms


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

    def init_exact_second_order_(self) -> None:
        """`LayerPredictor.init_exact_second_order_` on every layer."""
        for layer in self.layers:
            layer.init_exact_second_order_()

    def init_low_rank_second_order_(self, c_u: torch.Tensor,
                                    c_v: torch.Tensor,
                                    floor: float = 1e-6) -> None:
        """Per layer from moments [num_layers, num_heads, D, D]
        (predictor.py:367-385)."""
        if c_u.shape[0] != len(self.layers) or c_v.shape[0] != len(
                self.layers):
            raise ValueError('one moment per layer is needed')
        for index, layer in enumerate(self.layers):
            layer.init_low_rank_second_order_(c_u[index], c_v[index], floor)

    def scores(self, layer: int, q_tiles: torch.Tensor, k_tiles: torch.Tensor,
               layout: tiling.TileLayout, heads: torch.Tensor) -> torch.Tensor:
        """Block logits of one head group [H', n, n] fp32, with the
        optional terms' inputs pooled from the same tiles
        (predictor.py:387-410)."""
        feats_q = pool_tiles(q_tiles, layout)
        feats_k = pool_tiles(k_tiles, layout)
        extra = {}
        if self.count_term:
            extra['log_count'] = log_tile_counts(layout)
        if self.second_order_rank:
            extra['sq_q'] = pool_tiles(q_tiles, layout, SECOND_RAW)
            extra['var_k'] = pool_tiles(k_tiles, layout, SECOND_CENTRAL)
        return self.layers[layer](feats_q, feats_k, heads, **extra)


def log_tile_counts(layout: tiling.TileLayout) -> torch.Tensor:
    """[n_tiles] fp32 log of each tile's real rows, clamped to >= 1: the
    count term's input (attention.py:278-280)."""
    return torch.log(layout.valid_count.clamp(min=1).to(torch.float32))
