"""The block-sparse attention backend: drop-in for the reference's
`miowtion/kernels/fa4.py` (same function names, argument meaning, tensor
layouts and errors), backed by the sm_100a kernels of this package.

    from miowtion_b200 import kernels as fa4

q, k, v are tile-ordered [N, H', D] bf16 (the reference's FA4-native
seq-major layout). Block patterns are dense block masks [H', R, n] bool, or
the full/partial index lists of `mask.select_block_lists`, which the hot
path passes straight through. There is no fallback: without a B200 and the
built library every entry point raises.
"""

from __future__ import annotations

import heapq
import math
import threading

import torch

from miowtion_b200 import _lib
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import tiling

_TILE = tiling.TILE_SIZE
# Host launches are stateless and thread-safe; the lock only mirrors the
# reference's serialization point (fa4.py:66-70) for callers that rely on it.
_CALL_LOCK = threading.Lock()


def available(device: torch.device | None = None) -> bool:
    """True on a CUDA sm_100 device with the library built (fa4.py:122-137)."""
    return unavailable_reason(device) is None


def unavailable_reason(device: torch.device | None = None,
                       dtype: torch.dtype | None = None) -> str | None:
    """Why the kernels cannot run on `device`, or None (fa4.py:150-182)."""
    if not torch.cuda.is_available():
        return 'no CUDA device'
    if device is not None and torch.device(device).type != 'cuda':
        return f'device {device} is not CUDA'
    if dtype is not None and dtype != torch.bfloat16:
        return f'the kernels take bf16, not {dtype}'
    major, minor = torch.cuda.get_device_capability(device)
    if (major, minor) != (10, 0):
        return (f'sm_{major}{minor} has no tcgen05 tensor cores; the kernels '
                'are built for sm_100a (B200)')
    try:
        _lib.load()
    except RuntimeError as e:
        return str(e)
    return None


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    scale: float, return_lse: bool, used: int | None = None
                    ) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Dense attention. q, k, v: [S, H, D] -> out [S, H, D], lse [S, H]
    (fa4.py:185-205). `used` restricts attention to rows [0, used) with
    zero outputs (and lse) on the rest (h3/attention.py:28-102)."""
    _require(q, 'dense_attention')
    seq_len, heads, dim = q.shape
    used = seq_len if used is None else used
    for t in (k, v):
        if t.shape != q.shape or t.stride() != q.stride():
            raise ValueError('q, k and v must share shape and strides')
    out = torch.empty_like(q)
    lse = (torch.empty(seq_len, heads, dtype=torch.float32, device=q.device)
           if return_lse else None)
    _lib.call('veda_dense_fwd', q.data_ptr(), k.data_ptr(), v.data_ptr(),
              q.stride(0), q.stride(1), seq_len, used, heads, out.data_ptr(),
              out.stride(0), out.stride(1), _lib.ptr(lse),
              lse.stride(0) if lse is not None else 0,
              lse.stride(1) if lse is not None else 0, float(scale),
              _lib.stream_ptr(q.device))
    return out, lse


def index_lists(block_mask: torch.Tensor, layout: tiling.TileLayout,
                transpose: bool = False) -> tuple[torch.Tensor, ...]:
    """Full / partial index lists (fa4.py:275-296):
    (partial_cnt, partial_idx, full_cnt, full_idx), cnt [1, H', rows] and
    idx [1, H', rows, cols] int32, bit-identical to the reference's
    (members ascending, then the non-members ascending)."""
    lists = _lists(block_mask, layout, transpose=transpose, tails=True)
    return lists.as_fa4()


def _lists(block_mask: torch.Tensor, layout: tiling.TileLayout,
           transpose: bool, tails: bool) -> veda_mask.BlockLists:
    if block_mask.dim() != 3 or block_mask.shape[2] != layout.n_tiles:
        raise ValueError('block_mask must be [H\', R, n_tiles]')
    if not block_mask.is_cuda:
        raise RuntimeError('index_lists runs on CUDA only (no CPU fallback)')
    heads, rows, cols = block_mask.shape
    if transpose and rows != layout.n_tiles:
        raise ValueError('transposed lists need all n_tiles query rows')
    m = block_mask.to(torch.uint8).contiguous()
    out_rows, out_cols = (cols, rows) if transpose else (rows, cols)
    dev = block_mask.device
    lists = veda_mask.BlockLists(
        part_cnt=torch.empty(heads, out_rows, dtype=torch.int32, device=dev),
        part_idx=torch.empty(heads, out_rows, out_cols, dtype=torch.int32,
                             device=dev),
        full_cnt=torch.empty(heads, out_rows, dtype=torch.int32, device=dev),
        full_idx=torch.empty(heads, out_rows, out_cols, dtype=torch.int32,
                             device=dev))
    _lib.call('veda_index_lists', m.data_ptr(), heads, rows, cols,
              layout.valid_count.data_ptr(), 1 if transpose else 0,
              lists.part_cnt.data_ptr(), lists.part_idx.data_ptr(),
              lists.full_cnt.data_ptr(), lists.full_idx.data_ptr(),
              1 if tails else 0, _lib.stream_ptr(dev))
    return lists


def index_lists_from_mask(mask: torch.Tensor, layout: tiling.TileLayout,
                          transpose: bool = True) -> veda_mask.BlockLists:
    """Lists of a uint8 or bool block mask [H', n, n] (the mask
    `select_block_lists(..., want_mask=True)` returns), by default the
    transposed ones the backward walks."""
    return _lists(mask.bool() if mask.dtype != torch.bool else mask, layout,
                  transpose=transpose, tails=False)


def _require(q: torch.Tensor, op: str) -> None:
    reason = unavailable_reason(q.device, q.dtype)
    if reason is not None:
        raise NotImplementedError(
            f'{op} unavailable on {q.device}: {reason}; refusing to fall back '
            'to dense attention')


def block_sparse_attention_lists(q: torch.Tensor, k: torch.Tensor,
                                 v: torch.Tensor,
                                 lists: veda_mask.BlockLists,
                                 layout: tiling.TileLayout,
                                 return_lse: bool = False):
    """Forward over prebuilt lists (rows of `lists` = query tiles of q)."""
    _require(q, 'block_sparse_attention')
    for name, t in (('q', q), ('k', k), ('v', v)):
        tiling._check_rows(t, name)  # pylint: disable=protected-access
    heads = q.shape[1]
    n_q = q.shape[0] // _TILE
    if q.shape[0] != n_q * _TILE or k.shape[0] != layout.num_slots or (
            v.shape != k.shape):
        raise ValueError('q must hold whole tiles; k, v all key tiles')
    if lists.part_cnt.shape != (heads, n_q):
        raise ValueError(f'lists cover {tuple(lists.part_cnt.shape)} '
                         f'(heads, query tiles), expected {(heads, n_q)}')
    out = torch.empty_like(q)
    lse = (torch.empty(heads, n_q * _TILE, dtype=torch.float32,
                       device=q.device) if return_lse else None)
    _lib.call('veda_bsa_fwd', q.data_ptr(), q.stride(0), q.stride(1),
              k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(),
              v.stride(0), v.stride(1), heads, n_q, layout.n_tiles,
              layout.valid_count.data_ptr(), lists.part_cnt.data_ptr(),
              lists.part_idx.data_ptr(), lists.full_cnt.data_ptr(),
              lists.full_idx.data_ptr(), lists.part_idx.shape[-1],
              out.data_ptr(), out.stride(0), out.stride(1), _lib.ptr(lse),
              1.0 / math.sqrt(q.shape[-1]), _lib.stream_ptr(q.device))
    return (out, lse) if return_lse else out


# Video spans the packed forward reads in place (one tensor map each).
PACKED_MAX_SPANS = 2


def packed_supported(layout: tiling.TileLayout) -> bool:
    """Whether `block_sparse_attention_packed` can run this layout."""
    return 1 <= len(layout.spans) <= PACKED_MAX_SPANS


_SM_RESERVE = 0


def set_sm_reserve(n: int) -> None:
    """veda_set_sm_reserve: leave `n` SMs free of the attention forward
    (for kernels that overlap it, such as NCCL collectives)."""
    global _SM_RESERVE
    _lib.call('veda_set_sm_reserve', n)
    _SM_RESERVE = n


DEFAULT_FWD_GROUPS = 2


def set_fwd_groups(groups: int) -> None:
    """veda_set_fwd_groups: the forward's softmax in two groups of warps on
    alternate key blocks (2, the default) or one group (1)."""
    _lib.call('veda_set_fwd_groups', groups)


def work_order(layout: tiling.TileLayout, n_heads: int,
               blocks: list[veda_mask.ColumnBlock],
               device: torch.device) -> torch.Tensor | None:
    """A balanced work order for the forward over the selection lists of
    `blocks` (cached on the layout), or None where the default order is
    balanced already (no global query rows, or fewer items than SMs).

    A global (text) query row keeps every non-empty key tile, about ten
    times a video row's budget, so striding items over the CTAs in order
    leaves some CTAs with two of them: 5 % above the mean at config 3 on
    one GPU, 18 % with six heads per GPU. Here the global rows are dealt
    first, then the video rows head by head, each to the CTA with the
    least work so far (heads stay together in time, so their key tiles
    stay in L2). Layout [rounds, G] int32, slot h * n_tiles + qt or -1.
    """
    n_global = layout.n_global_tiles
    sms = max(1, torch.cuda.get_device_properties(device).multi_processor_count
              - _SM_RESERVE)
    n_items = n_heads * layout.n_tiles
    if n_global == 0 or n_items <= sms:
        return None
    key = (n_heads, sms, tuple((b.start, b.stop, b.budget, b.real_tokens)
                               for b in blocks))
    cache = layout.work_orders
    if key in cache:
        return cache[key]
    valid = layout.valid_count.cpu().tolist()
    n_video = layout.n_video_tiles
    live_global_cols = sum(1 for c in range(n_video, layout.n_tiles)
                           if valid[c] > 0)
    per_row = 0.0
    for arr in veda_mask.resolve_blocks(blocks):
        per_row += (arr.k_lo + arr.frac) if not arr.keeps_all else arr.k_lo
    video_weight = per_row + live_global_cols
    global_weight = float(sum(1 for v in valid if v > 0))
    order = balanced_order(n_heads, layout.n_tiles, n_video, global_weight,
                           video_weight, sms).to(device)
    cache[key] = order
    return order


def balanced_order(n_heads: int, n_tiles: int, n_video: int,
                   global_weight: float, video_weight: float,
                   ctas: int) -> torch.Tensor:
    """The work order of `work_order` on the host: the global query rows
    (tiles >= n_video) of every head first, then the video rows head by
    head (each head's tiles in reverse), every item to the CTA with the
    least work so far (ties to the lower CTA). [rounds, ctas] int32 with
    slots h * n_tiles + qt, -1 where a CTA has no more items."""
    heavy = [(h, qt) for h in range(n_heads)
             for qt in range(n_tiles - 1, n_video - 1, -1)]
    light = [(h, qt) for h in range(n_heads)
             for qt in range(n_video - 1, -1, -1)]
    loads = [(0.0, c) for c in range(ctas)]
    lists = [[] for _ in range(ctas)]
    for items, weight in ((heavy, global_weight), (light, video_weight)):
        for h, qt in items:
            load, c = heapq.heappop(loads)
            lists[c].append(h * n_tiles + qt)
            heapq.heappush(loads, (load + weight, c))
    rounds = max(len(x) for x in lists)
    order = torch.full((rounds, ctas), -1, dtype=torch.int32)
    for c, items in enumerate(lists):
        if items:
            order[:len(items), c] = torch.tensor(items, dtype=torch.int32)
    return order


def block_sparse_attention_packed(q: torch.Tensor, k: torch.Tensor,
                                  v: torch.Tensor,
                                  lists: veda_mask.BlockLists,
                                  layout: tiling.TileLayout,
                                  heads: torch.Tensor,
                                  out: torch.Tensor,
                                  kv_tiles: bool = False,
                                  order: torch.Tensor | None = None) -> None:
    """Forward of the heads `heads` of one tile layout, with the queries
    read from and the output written to the packed tensors in place:
    q [S, H, D] -> rows [0, used) of out [S, H, D] for those heads. Equals
    `gather_tiles`, then `block_sparse_attention_lists` over all query
    tiles, then `scatter_rows_` (veda/attention.py:724-743), in one kernel
    without the tile-ordered q or output. `order` (see `work_order`) only
    balances the CTAs' work. k and v are the group's
    tile-ordered copies [N, H', D] with `kv_tiles` (as `gather_and_pool`
    writes them), else packed [S, H, D] like q and read in place too."""
    _require(q, 'block_sparse_attention')
    for name, t in ((('q', q), ('out', out)) if kv_tiles == 'images' else
                    (('q', q), ('k', k), ('v', v), ('out', out))):
        tiling._check_rows(t, name)  # pylint: disable=protected-access
    if kv_tiles == 'images' and (k.dtype != torch.bfloat16
                                 or v.dtype != torch.bfloat16):
        raise NotImplementedError('tile images hold bf16')
    if not packed_supported(layout):
        raise ValueError(f'the packed forward reads at most '
                         f'{PACKED_MAX_SPANS} spans, the layout has '
                         f'{len(layout.spans)}')
    heads = tiling._heads_arg(q, heads)  # pylint: disable=protected-access
    n_heads = heads.numel()
    if out.shape != q.shape:
        raise ValueError('q and out must share [S, H, D]')
    if kv_tiles == 'images':
        if k.shape != (n_heads, layout.n_tiles, 2, 128, 64) or (
                v.shape != k.shape) or not (k.is_contiguous()
                                            and v.is_contiguous()):
            raise ValueError('tile images must be [len(heads), n_tiles, 2, '
                             '128, 64] contiguous')
    elif kv_tiles:
        if k.shape != (layout.num_slots, n_heads, q.shape[-1]) or (
                v.shape != k.shape or v.stride() != k.stride()):
            raise ValueError('tile-ordered k and v must be [num_slots, '
                             'len(heads), D] with equal strides')
    elif k.shape != q.shape or v.shape != q.shape or (
            k.stride() != q.stride() or v.stride() != q.stride()):
        raise ValueError('packed q, k and v must share [S, H, D] and strides')
    if lists.part_cnt.shape != (n_heads, layout.n_tiles):
        raise ValueError(f'lists cover {tuple(lists.part_cnt.shape)} '
                         f'(heads, query tiles), expected '
                         f'{(n_heads, layout.n_tiles)}')
    glob = [None, None, None]
    if layout.n_global_tiles:
        rows = torch.arange(layout.n_video_tiles, layout.n_tiles,
                            device=q.device)
        glob = [tiling.gather_tile_rows(t, layout, rows, heads)
                for t in ((q,) if kv_tiles else (q, k, v))]
        glob += [None] * (3 - len(glob))
    g_stride = glob[0].stride() if glob[0] is not None else (0, 0)
    _lib.call('veda_bsa_fwd_packed', q.data_ptr(), k.data_ptr(),
              v.data_ptr(), q.stride(0), q.stride(1), q.shape[0], q.shape[1],
              2 if kv_tiles == 'images' else (1 if kv_tiles else 0),
              k.stride(0), k.stride(1),
              *(_lib.ptr(t) for t in glob), g_stride[0], g_stride[1],
              tiling.span_array(layout.spans), len(layout.spans),
              layout.n_tiles, layout.n_video_tiles, heads.data_ptr(), n_heads,
              layout.box_perm.data_ptr(), layout.key_mask.data_ptr(),
              layout.valid_count.data_ptr(),
              lists.part_cnt.data_ptr(), lists.part_idx.data_ptr(),
              lists.full_cnt.data_ptr(), lists.full_idx.data_ptr(),
              lists.part_idx.shape[-1], out.data_ptr(), out.stride(0),
              out.stride(1), 1.0 / math.sqrt(q.shape[-1]),
              _lib.ptr(order), order.shape[1] if order is not None else 0,
              order.numel() if order is not None else 0,
              _lib.stream_ptr(q.device))


def block_sparse_attention_bwd(q: torch.Tensor, k: torch.Tensor,
                               v: torch.Tensor, out: torch.Tensor,
                               dout: torch.Tensor, lse: torch.Tensor,
                               lists: veda_mask.BlockLists,
                               t_lists: veda_mask.BlockLists,
                               layout: tiling.TileLayout
                               ) -> tuple[torch.Tensor, ...]:
    """dq, dk, dv of `block_sparse_attention_lists` (the backward FA4 runs
    through autograd, fa4.py:337-359). `lists` are the forward lists (per
    query tile), `t_lists` the transposed ones (per key tile,
    `index_lists(..., transpose=True)`); `lse` [H', R * 128] as the forward
    returned it. Rows of tiles without any block get zero gradients."""
    _require(q, 'block_sparse_attention backward')
    heads = q.shape[1]
    n_q = q.shape[0] // _TILE
    if t_lists.part_cnt.shape != (heads, layout.n_tiles):
        raise ValueError('transposed lists must cover every key tile')
    dout = dout if dout.stride(-1) == 1 and dout.stride(0) % 8 == 0 and (
        dout.stride(1) % 8 == 0) else dout.contiguous()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    need = _lib.load().veda_bsa_bwd_workspace(heads, n_q)
    ws = torch.empty(max(need, 16) // 4, dtype=torch.float32, device=q.device)
    _lib.call('veda_bsa_bwd', q.data_ptr(), q.stride(0), q.stride(1),
              k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(),
              v.stride(0), v.stride(1), out.data_ptr(), out.stride(0),
              out.stride(1), dout.data_ptr(), dout.stride(0), dout.stride(1),
              lse.data_ptr(), lse.stride(1), lse.stride(0), heads, n_q,
              layout.n_tiles, layout.valid_count.data_ptr(),
              lists.part_cnt.data_ptr(), lists.part_idx.data_ptr(),
              lists.full_cnt.data_ptr(), lists.full_idx.data_ptr(),
              lists.part_idx.shape[-1], t_lists.part_cnt.data_ptr(),
              t_lists.part_idx.data_ptr(), t_lists.full_cnt.data_ptr(),
              t_lists.full_idx.data_ptr(), t_lists.part_idx.shape[-1],
              dq.data_ptr(), dq.stride(0), dq.stride(1), dk.data_ptr(),
              dk.stride(0), dk.stride(1), dv.data_ptr(), dv.stride(0),
              dv.stride(1), 1.0 / math.sqrt(q.shape[-1]), ws.data_ptr(),
              ws.numel() * 4, _lib.stream_ptr(q.device))
    return dq, dk, dv


class _BlockSparseAttention(torch.autograd.Function):
    """Forward and backward over prebuilt forward and transposed lists."""

    @staticmethod
    def forward(ctx, q, k, v, lists, t_lists, layout):
        out, lse = block_sparse_attention_lists(q, k, v, lists, layout,
                                                return_lse=True)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.lists, ctx.t_lists, ctx.layout = lists, t_lists, layout
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, dout, _dlse):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = block_sparse_attention_bwd(q, k, v, out, dout, lse,
                                                ctx.lists, ctx.t_lists,
                                                ctx.layout)
        return dq, dk, dv, None, None, None


def block_sparse_attention_autograd(q: torch.Tensor, k: torch.Tensor,
                                    v: torch.Tensor,
                                    lists: veda_mask.BlockLists,
                                    t_lists: veda_mask.BlockLists,
                                    layout: tiling.TileLayout):
    """(out, lse) with gradients for q, k, v (both list directions given)."""
    return _BlockSparseAttention.apply(q, k, v, lists, t_lists, layout)


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           block_mask: torch.Tensor,
                           layout: tiling.TileLayout,
                           return_lse: bool = False):
    """Block-sparse attention on tile-ordered tensors (fa4.py:299-377).

    Args:
        q: [R * 128, H', D] bf16 query tiles (all tiles, or the subset whose
            rows `block_mask` describes).
        k, v: [N, H', D] bf16 (all key tiles).
        block_mask: [H', R, n_tiles] bool; empty key tiles are skipped.
        layout: Tile layout (valid prefix of every key tile).
        return_lse: Also return the [H', R * 128] fp32 log-sum-exp.

    Raises:
        NotImplementedError: Off B200 (no fallback).
        ValueError: If gradients are required for a subset of query tiles.
    """
    _require(q, 'block_sparse_attention')
    needs_grad = torch.is_grad_enabled() and any(
        t.requires_grad for t in (q, k, v))
    if needs_grad and block_mask.shape[1] != layout.n_tiles:
        raise ValueError('backward needs the block mask of all query tiles')
    lists = _lists(block_mask, layout, transpose=False, tails=False)
    with _CALL_LOCK:
        if needs_grad:
            # The backward walks key-tile-major lists (fa4.py:353-359).
            t_lists = _lists(block_mask, layout, transpose=True, tails=False)
            out, lse = _BlockSparseAttention.apply(q, k, v, lists, t_lists,
                                                   layout)
            return (out, lse) if return_lse else out
        return block_sparse_attention_lists(q, k, v, lists, layout,
                                            return_lse)
