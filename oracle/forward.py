"""CPU oracle for the Shrimp serve forward — TEST INFRASTRUCTURE ONLY.

This module is the checker the CUDA path is compared against. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import it; the
product path (hexo_bot_b200) never does, and it never runs on the GPU.

It restates, in plain fp32 torch on CPU, the reference network's serve path
over a state_dict with the reference parameter names:

- trunk                   packages/shrimp/python/shrimp/model.py:851-929
- HexNodeConv.forward     model.py:346-370
- ConvBlock.forward       model.py:395-422 (eager branch, :419-422)
- _build_pair             model.py:677-716
- build_attn_bias         model.py:718-760 (no-grad branch: fp16 table)
- RelPosAttention.forward model.py:448-492 ("sdpa" impl, :486-492)
- AttnBlock.forward       model.py:508-514
- _pooled / _value_input  model.py:931-935, 1005-1009
- forward_policy_value    model.py:972-1003
- _policy_logits          model.py:1011-1020
- decode_binned_value     packages/shrimp/python/shrimp/losses.py:40-51
- legal-prefix softmax    packages/shrimp/python/shrimp/inference.py:998-1042

Parity is pinned against outputs of the reference itself, generated in the
build container by tests/golden/make_golden.py (tests/test_oracle_golden.py).
"""

from __future__ import annotations

import math

import numpy as np
import torch
from torch.nn import functional as F

NUM_TOKENS = 8
VALUE_BINS = 65
BIAS_ROWS = 237
TOKEN_TOKEN, TOKEN_CELL, CELL_TOKEN = 236, 235, 234
PAD_KEY = -3.0e4
LN_EPS = 1e-5


# --- index tables ---------------------------------------------------------------


def _hex_dist(dq, dr):
    return max(abs(dq), abs(dr), abs(dq + dr))


def rel_bias_row(dq: int, dr: int) -> int:
    """packages/shrimp/python/shrimp/geometry.py:115-131, restated."""

    d = _hex_dist(dq, dr)
    if d <= 8:
        order = [(a, b) for a in range(-8, 9) for b in range(-8, 9) if _hex_dist(a, b) <= 8]
        return order.index((dq, dr))
    if d <= 16:
        on_axis = dq == 0 or dr == 0 or dq + dr == 0
        return (217 if on_axis else 225) + d - 9
    return 233


def cell_lut() -> np.ndarray:
    """35x35 row LUT over clamped offsets (model.py:625-641)."""

    m, w = 17, 35
    lut = np.zeros(w * w, dtype=np.int64)
    exact = {}
    k = 0
    for a in range(-8, 9):
        for b in range(-8, 9):
            if _hex_dist(a, b) <= 8:
                exact[(a, b)] = k
                k += 1
    for dq in range(-m, m + 1):
        for dr in range(-m, m + 1):
            d = _hex_dist(dq, dr)
            if d <= 8:
                row = exact[(dq, dr)]
            elif d <= 16:
                row = (217 if (dq == 0 or dr == 0 or dq + dr == 0) else 225) + d - 9
            else:
                row = 233
            lut[(dq + m) * w + dr + m] = row
    return lut


_LUT = torch.from_numpy(cell_lut())


def build_pair(coords: torch.Tensor, mask: torch.Tensor):
    """(pair (B,S,S) int64, key_live (B,S) bool) per model.py:677-716."""

    b, n, _ = coords.shape
    c = coords.to(torch.int64)
    dq = c[:, None, :, 0] - c[:, :, None, 0]
    dr = c[:, None, :, 1] - c[:, :, None, 1]
    idx = (dq.clamp(-17, 17) + 17) * 35 + (dr.clamp(-17, 17) + 17)
    cell = _LUT[idx.reshape(-1)].reshape(b, n, n)
    s = NUM_TOKENS + n
    pair = torch.full((b, s, s), TOKEN_TOKEN, dtype=torch.int64)
    pair[:, :NUM_TOKENS, NUM_TOKENS:] = TOKEN_CELL
    pair[:, NUM_TOKENS:, :NUM_TOKENS] = CELL_TOKEN
    pair[:, NUM_TOKENS:, NUM_TOKENS:] = cell
    key_live = torch.cat([torch.ones(b, NUM_TOKENS, dtype=torch.bool), mask.to(torch.bool)], dim=1)
    return pair, key_live


def build_pair_u8(coords: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """(B,S,S) uint8 pair rows with dead keys -> row 237 (model.py:762-792)."""

    pair, key_live = build_pair(coords, mask)
    pair = pair.masked_fill(~key_live[:, None, :], BIAS_ROWS)
    return pair.to(torch.uint8)


def gather_index(nbr: torch.Tensor) -> torch.Tensor:
    """(B,Npad,7) int64: tap 0 = self, taps 1..6 = nbr (missing -> Npad)."""

    b, n, _ = nbr.shape
    self_idx = torch.arange(n).reshape(1, n, 1).expand(b, -1, -1)
    return torch.cat([self_idx, nbr.to(torch.int64)], dim=2)


# --- layers ---------------------------------------------------------------------


def hex_conv(x, gidx, mask, weight, bias):
    """Gather 7 taps (zero row at Npad) then one GEMM (model.py:366-370)."""

    b, n, c = x.shape
    x_ext = torch.cat([x, x.new_zeros(b, 1, c)], dim=1)
    taps = gidx.shape[2]
    flat = gidx.reshape(b, n * taps, 1).expand(-1, -1, c)
    g = x_ext.gather(1, flat).reshape(b, n, taps * c)
    out = g @ weight.reshape(taps * c, weight.shape[-1]) + bias
    return out * mask.unsqueeze(-1)


def layer_norm(x, w, b):
    return F.layer_norm(x, (x.shape[-1],), w, b, LN_EPS)


def linear(x, sd, name):
    return F.linear(x, sd[name + ".weight"], sd[name + ".bias"])


def conv_block(sd, p, x, gidx, mask):
    m = mask.unsqueeze(-1)
    y = F.relu(layer_norm(hex_conv(x, gidx, mask, sd[p + "conv1.weight"], sd[p + "conv1.bias"]),
                          sd[p + "ln1.weight"], sd[p + "ln1.bias"])) * m
    y = layer_norm(hex_conv(y, gidx, mask, sd[p + "conv2.weight"], sd[p + "conv2.bias"]),
                   sd[p + "ln2.weight"], sd[p + "ln2.bias"]) * m
    return F.relu(x + y * sd[p + "ls.gamma"])


def attn_bias(table, pair, key_live):
    """(B,H,S,S) additive bias; the table is rounded to fp16 first
    (model.py:737-760)."""

    bias_t = table.to(torch.float16).t().contiguous()
    bias = bias_t[:, pair].permute(1, 0, 2, 3)
    fill = torch.where(key_live, 0.0, PAD_KEY).to(bias.dtype)
    return bias + fill[:, None, None, :]


def rel_attention(sd, p, seq, bias, heads):
    b, s, c = seq.shape
    d = c // heads
    q = linear(seq, sd, p + "q_proj").reshape(b, s, heads, d).transpose(1, 2)
    k = linear(seq, sd, p + "k_proj").reshape(b, s, heads, d).transpose(1, 2)
    v = linear(seq, sd, p + "v_proj").reshape(b, s, heads, d).transpose(1, 2)
    out = F.scaled_dot_product_attention(q, k, v, attn_mask=bias.to(q.dtype))
    out = out.transpose(1, 2).reshape(b, s, c)
    return linear(out, sd, p + "out_proj")


def attn_block(sd, p, seq, bias, seq_mask, heads):
    m = seq_mask.unsqueeze(-1)
    a = rel_attention(sd, p + "attn.", layer_norm(seq, sd[p + "ln1.weight"], sd[p + "ln1.bias"]), bias, heads)
    seq = seq + a * m * sd[p + "ls_attn.gamma"]
    h = layer_norm(seq, sd[p + "ln2.weight"], sd[p + "ln2.bias"])
    u = linear(F.gelu(linear(h, sd, p + "fc1")), sd, p + "fc2")
    return seq + u * m * sd[p + "ls_mlp.gamma"]


def trunk(sd, feats, nbr, mask, coords, heads, layout):
    b, n, _ = feats.shape
    mask = mask.to(torch.bool)
    gidx = gather_index(nbr)
    mf = mask.unsqueeze(-1)
    x = F.relu(layer_norm(hex_conv(feats.float(), gidx, mask, sd["stem.weight"], sd["stem.bias"]),
                          sd["stem_ln.weight"], sd["stem_ln.bias"])) * mf
    pair, key_live = build_pair(coords, mask)
    seq_mask = torch.cat([torch.ones(b, NUM_TOKENS, dtype=torch.bool), mask], dim=1)
    tokens = sd["tokens"].unsqueeze(0).expand(b, -1, -1)
    ci = ai = 0
    seq = None
    for pos, kind in enumerate(layout):
        if kind == "C":
            x = conv_block(sd, f"conv_blocks.{ci}.", x, gidx, mask)
            ci += 1
        else:
            bias = attn_bias(sd[f"bias_tables.{ai}"], pair, key_live)
            seq = attn_block(sd, f"attn_blocks.{ai}.", torch.cat([tokens, x], dim=1), bias, seq_mask, heads)
            ai += 1
            if pos != len(layout) - 1:
                tokens, x = seq[:, :NUM_TOKENS], seq[:, NUM_TOKENS:]
    seq = layer_norm(seq, sd["ln_final.weight"], sd["ln_final.bias"])
    return seq[:, NUM_TOKENS:] * mf, seq[:, :NUM_TOKENS], gidx


def pooled(cells, mask):
    mask = mask.to(torch.bool)
    counts = mask.sum(dim=1, keepdim=True).clamp(min=1).to(cells.dtype)
    return (cells * mask.unsqueeze(-1)).sum(dim=1) / counts


@torch.no_grad()
def forward_policy_value(sd, feats, nbr, mask, coords, *, heads, layout, request_moves_left=False):
    """Reference serve outputs: {'policy' (B,Npad), 'value' (B,65)[, 'moves_left']}."""

    sd = {k: v.detach().float().cpu() for k, v in sd.items()}
    mask = mask.to(torch.bool).cpu()
    cells, tokens, gidx = trunk(sd, feats.cpu(), nbr.cpu(), mask, coords.cpu(), heads, layout)
    pool = pooled(cells, mask)
    y = F.relu(hex_conv(cells, gidx, mask, sd["policy_conv.weight"], sd["policy_conv.bias"]))
    policy = linear(y, sd, "policy_head").squeeze(-1) * mask
    vin = torch.cat([tokens[:, 0], tokens[:, 1], pool], dim=1)
    value = linear(F.relu(linear(vin, sd, "value_reduction")), sd, "value_head")
    out = {"policy": policy, "value": value}
    if request_moves_left:
        mlin = torch.cat([tokens[:, 4], tokens[:, 5], pool], dim=1)
        out["moves_left"] = linear(F.relu(linear(mlin, sd, "ml_reduction")), sd, "moves_left_head")
    return out


def decode_binned_value(logits: torch.Tensor) -> torch.Tensor:
    bins = torch.linspace(-1.0, 1.0, VALUE_BINS, dtype=logits.dtype)
    return (torch.softmax(logits, dim=-1) * bins).sum(dim=-1).clamp(-1.0, 1.0)


def legal_prefix_priors(policy: torch.Tensor, legal_counts) -> list[torch.Tensor]:
    """Per row: softmax over the first legal_counts[b] logits (inference.py:998-1042)."""

    out = []
    for b in range(policy.shape[0]):
        n = int(legal_counts[b])
        out.append(torch.softmax(policy[b, :n].float(), dim=0))
    return out


# --- microbench oracles (no reference implementation; HexNodeConv / materialized
# attention generalised, model.py:366-370 and :486-488) ---------------------------


def raytap_conv(x, nbr, weight, bias):
    """relu(gather-GEMM + bias + x): x (B,N,C), nbr (N,T) int (-1 -> zero row),
    weight (T*C, C) — the 19-tap microbench."""

    b, n, c = x.shape
    taps = nbr.shape[1]
    x_ext = torch.cat([x, x.new_zeros(b, 1, c)], dim=1)
    idx = torch.where(nbr >= 0, nbr, torch.full_like(nbr, n)).to(torch.int64)
    g = x_ext[:, idx.reshape(-1)].reshape(b, n, taps * c)
    return F.relu(g @ weight + bias + x)


def offset_bias_attention(q, k, v, table, offset_map, heads):
    """softmax(QK^T/sqrt(d) + table[offset_map, h]) V over (B, L, H*d) inputs."""

    b, l, hd = q.shape
    d = hd // heads
    qh = q.reshape(b, l, heads, d).transpose(1, 2)
    kh = k.reshape(b, l, heads, d).transpose(1, 2)
    vh = v.reshape(b, l, heads, d).transpose(1, 2)
    bias = table[offset_map.to(torch.int64)].permute(2, 0, 1)  # (H, L, L)
    s = qh @ kh.transpose(-1, -2) / math.sqrt(d) + bias
    return (torch.softmax(s, dim=-1) @ vh).transpose(1, 2).reshape(b, l, hd)


def derandomize(sd: dict, seed: int = 11) -> dict:
    """Open every residual branch so parity tests exercise the trunk: LayerScale
    gammas = 1, bias tables ~ N(0, 0.5), out_proj / fc2 weights += 0.05 N(0, 1)
    (after tests/test_shrimp_model.py:45-57 and :328-340 of the reference).
    Returns a new state_dict; deterministic in `seed`."""

    g = torch.Generator().manual_seed(seed)
    out = {k: v.detach().clone() for k, v in sd.items()}
    for k in sorted(out):
        v = out[k]
        if k.endswith("attn.out_proj.weight") or (k.startswith("attn_blocks.") and k.endswith("fc2.weight")):
            out[k] = v + torch.randn(v.shape, generator=g, dtype=torch.float32).to(v.dtype) * 0.05
        elif k.endswith(".gamma"):
            out[k] = torch.ones_like(v)
        elif k.startswith("bias_tables."):
            out[k] = torch.randn(v.shape, generator=g, dtype=torch.float32).to(v.dtype) * 0.5
    return out


def state_checksum(sd: dict) -> dict:
    """Per-tensor (sum, sum of squares) in float64 — a compact weight fingerprint."""

    return {k: (float(v.double().sum()), float(v.double().square().sum())) for k, v in sd.items()}
