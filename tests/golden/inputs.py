"""Seeded inputs and case specs shared by the golden generator and the tests.

Everything here uses torch's CPU generator, so the same seeds give the same
tensors in the build container (where the fixtures are made) and on the GPU
box (where the GPU tests regenerate them).
"""

from __future__ import annotations

import torch

# Config 1 of the benchmark: one CPU-runnable Veda layer (B=1, 8 heads,
# head_dim 128, grid (4,16,16) = 1024 tokens, tile (2,8,8), 50% budget).
CFG1 = dict(seq_len=1024, used=1024, heads=8, dim=128, seed=0,
            grid=(4, 16, 16), shape=(2, 8, 8), ratio=0.5, pred_seed=100,
            pred_std=0.02)

# A padded target grid behind text rows: partial tiles, a partial global
# tile and padding rows [used, seq_len). Small head_dim keeps fixtures tiny;
# the oracle does not depend on head_dim.
PADDED = dict(spans=[(360, (8, 12, 20), (4, 8, 4))], used=2280,
              seq_len=2312, heads=3, dim=32, seed=5, group_heads=[0, 2],
              pred_seed=101, ratio=0.3, score_seed=7, dout_seed=9,
              heat_rows=[0, 3, 7, 19, 22])

# Reference (condition) span + target span: segmented budgets.
SEGMENTED = dict(spans=[(90, (1, 16, 32), (1, 8, 16)),
                        (90 + 512 + 40, (16, 8, 16), (4, 8, 4))],
                 used=90 + 512 + 40 + 2048, seq_len=90 + 512 + 40 + 2048,
                 heads=3, ref_ratio=0.25, target_ratio=0.3, score_seed=11,
                 subset_rows=[0, 3, 4, 7, 11, 19])

# Layouts of the reference's own tiling tests (tests/unit/
# test_veda_tiling_plan.py:24-35): text 100, optional condition, audio 50.
SMALL_LAYOUTS = {
    'l_4x8x4': dict(spans=[(150, (7, 6, 10), (4, 8, 4))], used=570,
                    seq_len=600),
    'l_8x2x8': dict(spans=[(150, (7, 6, 10), (8, 2, 8))], used=570,
                    seq_len=600),
    'l_2x8x8': dict(spans=[(150, (7, 6, 10), (2, 8, 8))], used=570,
                    seq_len=600),
    'l_cond': dict(spans=[(100, (1, 6, 10), (1, 8, 16)),
                          (210, (7, 6, 10), (4, 8, 4))], used=630,
                   seq_len=660),
    'l_ragged': dict(spans=[(0, (3, 5, 7), (2, 8, 8))], used=105,
                     seq_len=130),
}

# Full-size layouts of benchmark configs 2-4 (budgets: (ref, target) ratios).
BENCH_LAYOUTS = {
    'cfg2': dict(spans=[(0, (20, 32, 56), (2, 8, 8))], used=35840,
                 seq_len=35840, budgets=[(None, 0.1)]),
    'cfg3_a': dict(spans=[(1024, (26, 45, 80), (2, 8, 8))], used=94624,
                   seq_len=94624, budgets=[(None, 0.1)]),
    'cfg3_b': dict(spans=[(1024, (26, 45, 80), (1, 8, 16))], used=94624,
                   seq_len=94624, budgets=[(None, 0.1)]),
    'cfg4': dict(spans=[(0, (4, 45, 80), (2, 8, 8)),
                        (14400, (26, 45, 80), (2, 8, 8))], used=108000,
                 seq_len=108000, budgets=[(0.05, 0.1)]),
}


def qkv(seq_len, heads, dim, seed, dtype):
    """q, k, v ~ N(0, 1) drawn in that order from one seeded generator."""
    gen = torch.Generator().manual_seed(seed)
    return [torch.randn(seq_len, heads, dim, generator=gen).to(dtype)
            for _ in range(3)]


def predictor_weights(heads, dim, seed, std):
    """proj_q, proj_k [heads, 3*dim, dim] fp32 ~ N(0, std^2)."""
    gen = torch.Generator().manual_seed(seed)
    return [torch.randn(heads, 3 * dim, dim, generator=gen) * std
            for _ in range(2)]


def scores(heads, n_tiles, seed):
    """Random fp32 block scores [heads, n_tiles, n_tiles] (no ties)."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(heads, n_tiles, n_tiles, generator=gen)


def dout(shape, seed):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=gen).to(torch.bfloat16)


# Tile search (oracle relative error): text rows, a video grid that three
# candidate shapes tile differently, bf16 q/k/v, 3 heads of head_dim 128.
SEARCH = dict(text=200, grid=(4, 16, 24), seq_len=1760, used=1736, heads=3,
              dim=128, seed=13, ratio=0.3, query_tiles=5, sample_seed=2,
              candidates=[(2, 8, 8), (1, 8, 16), (4, 4, 8)],
              # Plan vote: entries of random tables over these candidates.
              vote_layers=3, vote_entries=4, vote_heads=5, vote_seed=21,
              vote_grid=(37, 24, 42),
              vote_candidates=['8x4x4', '2x8x8', '4x4x8', '4x8x4', '8x2x8',
                               '8x8x2'])


def search_rows(n_video: int, count: int, seed: int, layer: int = 0):
    """Sorted sampled video query tiles, the reference OracleScorer's rule
    (search.py:227-230)."""
    gen = torch.Generator().manual_seed(seed * 1000 + layer)
    rows = torch.randperm(n_video, generator=gen)
    return rows[:min(count, n_video)].sort().values


def vote_tables(spec):
    """Seeded [C, H] score tables per (entry, layer)."""
    gen = torch.Generator().manual_seed(spec['vote_seed'])
    return [[torch.rand(len(spec['vote_candidates']), spec['vote_heads'],
                        generator=gen)
             for _ in range(spec['vote_layers'])]
            for _ in range(spec['vote_entries'])]


# Zero-order compensation: the padded target grid behind text rows (partial
# tiles, a partial global tile), head_dim 128 (the kernel's), a random keep
# mask from block scores, and a fixed projection for row checksums.
COMPENSATION = dict(spans=[(360, (8, 12, 20), (4, 8, 4))], used=2280,
                    seq_len=2312, heads=3, dim=128, seed=31, score_seed=32,
                    ratio=0.3, proj_seed=33, full_tile=5)


def projection(dim, seed):
    """[dim] fp32 weights for per-row checksums out[r, h] . w."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(dim, generator=gen)


# TeacherCollector (stage 1): text rows, a padded target grid cut by two tile
# shapes over the heads, two layers; each case a heat reduction, a KL
# direction, a share of supervised query tiles and optionally the weights
# of the ablation losses added to the seer KL.
TEACHER = dict(text=130, grid=(4, 12, 20), seq_len=1100, heads=4, dim=128,
               seed=81, pred_seed=82, pred_std=0.02, layers=2,
               shapes=[(2, 8, 8), (1, 8, 16)], head_shape=[0, 1, 0, 1],
               ratio=0.4, gen_seed=7, grad_scale=0.5,
               cases={'max_fwd': ('max', 'forward', 0.5),
                      'sum_rev': ('sum', 'reverse', 1.0),
                      'sum_ablate': ('sum', 'forward', 0.5,
                                     dict(transport_weight=0.5,
                                          gauge_kl_weight=0.25,
                                          topk_weight=0.3))})

# The ablation losses (transport, gauge-fixed KL, oracle BCE) on seeded
# logits and heat over the padded layout: supervised rows, a budget that
# reaches well past the diagonal, temperatures of the transport loss.
LOSSES = dict(heads=3, rows=[0, 3, 7, 12, 19], ratio=0.5, seed=93,
              temperatures=[0.15, 0.5, 1e-4])


# The predictor's optional score terms: a head subset out of order, a
# rank-8 second-order head and the count term, over seeded pooled features
# of 37 query and 41 key tiles (some key tiles partly or wholly empty).
PREDICTOR_TERMS = dict(heads=4, dim=128, rank=8, n_q=37, n_k=41, seed=61,
                       sub_heads=[2, 0, 3])


def predictor_term_inputs(spec):
    """Seeded parameters and pooled inputs of the optional-terms case."""
    gen = torch.Generator().manual_seed(spec['seed'])
    heads, dim, rank = spec['heads'], spec['dim'], spec['rank']
    sub = torch.tensor(spec['sub_heads'], dtype=torch.int64)
    n_sub, n_q, n_k = sub.numel(), spec['n_q'], spec['n_k']

    def normal(*shape, std=1.0):
        return torch.randn(*shape, generator=gen) * std

    counts = torch.randint(0, 129, (n_k,), generator=gen)
    counts[:3] = torch.tensor([128, 0, 17])
    return {
        'heads': sub,
        'proj_q': normal(heads, 3 * dim, dim, std=0.02),
        'proj_k': normal(heads, 3 * dim, dim, std=0.02),
        'so_q': normal(heads, dim, rank, std=0.05),
        'so_k': normal(heads, dim, rank, std=0.05),
        'count_gain': 1.0 + normal(heads, std=0.3),
        'feats_q': normal(n_sub, n_q, 3 * dim),
        'feats_k': normal(n_sub, n_k, 3 * dim),
        'sq_q': normal(n_sub, n_q, dim).square(),
        'var_k': normal(n_sub, n_k, dim).square() * 0.5,
        'log_count': torch.log(counts.clamp(min=1).float()),
        'probe': normal(n_sub, n_q, n_k),
    }


def predictor_term_moments(spec):
    """Seeded PSD moments [2, D, D] (two heads) of non-negative features
    (the first rank deficient on purpose: 96 samples of 128 features)."""
    gen = torch.Generator().manual_seed(spec['seed'] + 1)
    heads, dim = 2, spec['dim']
    u = torch.randn(heads, 96, dim, generator=gen).square()
    v = torch.randn(heads, 160, dim, generator=gen).square()
    return (u.transpose(1, 2) @ u / 96.0, v.transpose(1, 2) @ v / 160.0)


# The 'threshold' budget rule: seeded scores on the padded and segmented
# layouts, and a row subset of the padded one.
THRESHOLD = dict(seed=67, rows=[0, 2, 5, 11, 17, 19])
