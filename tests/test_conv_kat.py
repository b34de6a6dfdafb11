"""HexNodeConv known-answer test: the 7-tap gather conv equals a dense 3x3
conv on the axial grid embedded at (r+20, q+20), tap (dq, dr) at kernel slot
(dr+1, dq+1), fp64 (restated from the reference's
tests/test_shrimp_model.py:81-136). Pins the oracle's conv."""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as Fn

from hexo_bot_b200 import constants as K
from hexo_bot_b200 import featurize as F
from oracle import forward as O


def test_hex_conv_equals_dense_grid_conv():
    torch.manual_seed(1)
    cin, cout = 8, 8
    sup = F.build_support([(0, 0), (1, 0), (0, 1), (2, -1), (1, 1), (-1, 2), (3, 0)], 8)
    n = sup.num_nodes
    w = torch.randn(7, cin, cout, dtype=torch.float64)
    b = torch.randn(cout, dtype=torch.float64)
    kernel = torch.zeros(cout, cin, 3, 3, dtype=torch.float64)
    kernel[:, :, 1, 1] = w[0].T
    for k, (dq, dr) in enumerate(K.DIRECTIONS):
        kernel[:, :, dr + 1, dq + 1] = w[k + 1].T
    feats = torch.randn(1, n, cin, dtype=torch.float64)
    grid = torch.zeros(1, cin, 41, 41, dtype=torch.float64)
    for row, (q, r) in enumerate(sup.coords.tolist()):
        grid[0, :, r + 20, q + 20] = feats[0, row]
    nbr = torch.from_numpy(np.where(sup.nbr >= 0, sup.nbr, n).astype(np.int64)).unsqueeze(0)
    gidx = O.gather_index(nbr)
    mine = O.hex_conv(feats, gidx, torch.ones(1, n, dtype=torch.bool), w, b)
    dense = Fn.conv2d(grid, kernel, bias=b, padding=1)
    for row, (q, r) in enumerate(sup.coords.tolist()):
        assert torch.allclose(mine[0, row], dense[0, :, r + 20, q + 20], atol=1e-12)
