"""Seeded synthetic NN inputs in the reference's input layout.

Layouts follow the reference backend's input buffers (`crates/katago-nn-burn/src/backend.rs:150-212`): spatial
`[N, C, 19, 19]` float32 (NCHW, C = 22 for model versions 8-17), global `[N, 19]`, meta `[N, 192]` for human-SL nets.
Channel 0 is the on-board mask (bin2onnx.py:1203-1206); a board smaller than 19x19 sits in the top-left corner.

Distribution (the reference's bench harness `crates/katago-nn-burn/examples/bench.rs:27-32`, narrowed to the
benchmark configs): plane 0 = mask; planes 1-2 = own / opponent stones, a stone on ~30% of the on-board points with
an even colour split, never both; every other plane 0; global features U(-1, 1); meta features U(0, 1) sparse.
`rich=True` also fills planes 3..C-1 with sparse on-board bits, so that every input channel carries data in tests.
"""

from __future__ import annotations

from typing import Sequence, Tuple

import numpy as np

POS_LEN = 19


def synthetic_inputs(n: int, seed: int, board_sizes: Sequence[int] = (19,), num_spatial: int = 22,
                     num_global: int = 19, num_meta: int = 0, rich: bool = False
                     ) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """(spatial [n,C,19,19], global [n,G], meta [n,M] (M may be 0), board size per row [n])."""
    rng = np.random.default_rng(seed)
    sizes = np.asarray(board_sizes)[rng.integers(0, len(board_sizes), size=n)]
    yy, xx = np.meshgrid(np.arange(POS_LEN), np.arange(POS_LEN), indexing="ij")
    mask = (yy[None] < sizes[:, None, None]) & (xx[None] < sizes[:, None, None])
    stone = (rng.random((n, POS_LEN, POS_LEN)) < 0.3) & mask
    white = rng.random((n, POS_LEN, POS_LEN)) < 0.5
    spatial = np.zeros((n, num_spatial, POS_LEN, POS_LEN), np.float32)
    spatial[:, 0] = mask
    spatial[:, 1] = stone & white
    spatial[:, 2] = stone & ~white
    if rich:
        extra = (rng.random((n, num_spatial - 3, POS_LEN, POS_LEN)) < 0.08) & mask[:, None]
        spatial[:, 3:] = extra
    glob = rng.uniform(-1.0, 1.0, size=(n, num_global)).astype(np.float32)
    meta = np.zeros((n, num_meta), np.float32)
    if num_meta:
        meta = (rng.random((n, num_meta)) < 0.2).astype(np.float32) * rng.uniform(0, 1, size=(n, num_meta)).astype(np.float32)
    return spatial, glob, meta, sizes.astype(np.int32)
