"""ShrimpNet on B200: the reference module tree, served by native sm_100a kernels.

The module keeps the reference network's constructor, parameter names, shapes
and initialisation (packages/shrimp/python/shrimp/model.py:327-669), so a
reference checkpoint loads with ``load_state_dict(strict=True)`` and the same
``torch.manual_seed`` produces the same weights. ``forward_policy_value``
(model.py:972-1003) runs entirely in the shrimp_b200 native library: one C-ABI
call enqueues the whole forward (stem, ConvBlocks, AttnBlocks, heads) on the
current CUDA stream. There is no CPU or eager fallback; CPU inputs raise.

Weights are packed once into kernel layouts (f16 K-major tensor-core operands,
fp32 epilogue vectors) and re-packed automatically when a parameter changes.
"""

from __future__ import annotations

import ctypes as C
import math

import torch
from torch import nn
from torch.nn import functional as F

from . import _lib
from . import constants as K
from .geometry import cell_bias_lut

STV_HORIZONS = (2, 6, 16)

KNOWN_TRUNK_LAYOUTS: dict[tuple[int, int], str] = {
    (8, 3): "CCCACCCACCA",
    (10, 5): "CCACCACCACCACCA",
}


class HexNodeConv(nn.Module):
    """Direction-typed 7-tap hex convolution parameters (model.py:327-370):
    weight (7, Cin, Cout) with tap 0 = self and taps 1..6 = DIRECTIONS, bias
    (Cout,), both U(+-1/sqrt(7 Cin))."""

    def __init__(self, in_channels: int, out_channels: int) -> None:
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.weight = nn.Parameter(torch.empty(7, in_channels, out_channels))
        self.bias = nn.Parameter(torch.empty(out_channels))
        bound = 1.0 / math.sqrt(7 * in_channels)
        nn.init.uniform_(self.weight, -bound, bound)
        nn.init.uniform_(self.bias, -bound, bound)


class LayerScale(nn.Module):
    """Per-channel residual scale gamma, initialised to 1e-4 (model.py:373-381)."""

    def __init__(self, channels: int, init: float = 1e-4) -> None:
        super().__init__()
        self.gamma = nn.Parameter(torch.full((channels,), init))


class ConvBlock(nn.Module):
    """conv1 -> LN -> ReLU -> mask -> conv2 -> LN -> mask -> x gamma + x -> ReLU
    (model.py:384-422)."""

    def __init__(self, channels: int) -> None:
        super().__init__()
        self.conv1 = HexNodeConv(channels, channels)
        self.ln1 = nn.LayerNorm(channels)
        self.conv2 = HexNodeConv(channels, channels)
        self.ln2 = nn.LayerNorm(channels)
        self.ls = LayerScale(channels)


class RelPosAttention(nn.Module):
    """q/k/v/out projections of the biased attention (model.py:425-446)."""

    def __init__(self, channels: int, heads: int | None = None) -> None:
        super().__init__()
        self.heads = K.ATTENTION_HEADS if heads is None else int(heads)
        self.head_dim = channels // self.heads
        self.scale = 1.0 / math.sqrt(self.head_dim)
        self.q_proj = nn.Linear(channels, channels)
        self.k_proj = nn.Linear(channels, channels)
        self.v_proj = nn.Linear(channels, channels)
        self.out_proj = nn.Linear(channels, channels)
        self.impl = "sdpa"


class AttnBlock(nn.Module):
    """Pre-norm transformer block over [tokens ; cells] (model.py:495-514)."""

    def __init__(self, channels: int, heads: int | None = None) -> None:
        super().__init__()
        self.ln1 = nn.LayerNorm(channels)
        self.attn = RelPosAttention(channels, heads)
        self.ln2 = nn.LayerNorm(channels)
        self.fc1 = nn.Linear(channels, K.MLP_RATIO * channels)
        self.fc2 = nn.Linear(K.MLP_RATIO * channels, channels)
        self.ls_attn = LayerScale(channels)
        self.ls_mlp = LayerScale(channels)


def infer_net_kwargs_from_state_dict(sd: dict) -> dict:
    """Constructor kwargs recovered from a checkpoint (model.py:529-555)."""

    kwargs: dict = {}
    for key, axis in (("stem.bias", 0), ("stem_ln.weight", 0), ("tokens", 1)):
        shape = getattr(sd.get(key), "shape", None)
        if shape is not None and len(shape) > axis:
            kwargs["channels"] = int(shape[axis])
            break
    bt = sd.get("bias_tables.0")
    if bt is not None and len(getattr(bt, "shape", ())) == 2:
        kwargs["attention_heads"] = int(bt.shape[1])
    conv_ids = {int(k.split(".")[1]) for k in sd if k.startswith("conv_blocks.")}
    attn_ids = {int(k.split(".")[1]) for k in sd if k.startswith("attn_blocks.")}
    if conv_ids and attn_ids:
        layout = KNOWN_TRUNK_LAYOUTS.get((max(conv_ids) + 1, max(attn_ids) + 1))
        if layout is not None:
            kwargs["trunk_layout"] = layout
    return kwargs


def _dtype_code(t: torch.Tensor) -> int:
    return {
        torch.float32: _lib.DT_F32,
        torch.float16: _lib.DT_F16,
        torch.bfloat16: _lib.DT_BF16,
        torch.int64: _lib.DT_I64,
        torch.int32: _lib.DT_I32,
        torch.uint8: _lib.DT_U8,
        torch.bool: _lib.DT_U8,
        torch.int16: _lib.DT_I16,
        torch.uint16: _lib.DT_U16,
    }[t.dtype]


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class PackedWeights:
    """Device-resident kernel-layout copy of a ShrimpNet's serve weights plus the
    C `sb_net` descriptor pointing into it.

    Construction allocates every buffer once; `refresh()` re-packs the current
    parameter values into those same buffers with device work only (no host
    copy, no synchronisation), so it may run inside CUDA-graph capture and a
    graph captured earlier keeps valid pointers. fp32 vectors that already
    live on the device as contiguous fp32 tensors are used in place."""

    def __init__(self, model: "ShrimpNet", device: torch.device) -> None:
        self.device = device
        self.keep: list[torch.Tensor] = []
        self._ops: list = []  # refresh steps, in order
        self.packed_in_capture = False
        c, h = model.channels, model.heads
        net = _lib.Net()
        net.channels = c
        net.heads = h
        net.num_blocks = len(model._trunk_layout)
        net.layout = model._trunk_layout.encode()

        def live(t: torch.Tensor) -> bool:
            return t.device == device and t.dtype == torch.float32 and t.is_contiguous()

        def f32(t: torch.Tensor) -> int:
            """fp32 copy (or the tensor itself when it already is one) of a
            parameter or of a view of one (e.g. a transpose)."""
            if live(t):
                self.keep.append(t)
                return t.data_ptr()
            buf = torch.empty(t.shape, dtype=torch.float32, device=device)
            self.keep.append(buf)
            self._ops.append(lambda t=t, buf=buf: buf.copy_(t.detach()))
            return buf.data_ptr()

        def stage(*parts: torch.Tensor) -> torch.Tensor:
            """fp32 device source of a pack kernel: the parameter itself, or a
            buffer refreshed from the (concatenated) parameters."""
            if len(parts) == 1 and live(parts[0]):
                return parts[0]
            n = sum(int(x.shape[0]) for x in parts)
            buf = torch.empty((n,) + tuple(parts[0].shape[1:]), dtype=torch.float32, device=device)
            self.keep.append(buf)

            def op(parts=parts, buf=buf):
                off = 0
                for x in parts:
                    buf[off:off + x.shape[0]].copy_(x.detach())
                    off += x.shape[0]
            self._ops.append(op)
            return buf

        def conv_w(mod: HexNodeConv, cin_pad: int) -> int:
            src = stage(mod.weight)
            kpad = _round_up(7 * cin_pad, 64)
            out = torch.empty(mod.out_channels, kpad, dtype=torch.float16, device=device)
            self.keep.append(out)

            def op(src=src, out=out, mod=mod):
                _lib.check(_lib.lib().sb_pack_hex_conv_weight(
                    src.data_ptr(), 7, mod.in_channels, cin_pad, mod.out_channels, out.data_ptr(),
                    torch.cuda.current_stream(device).cuda_stream), "sb_pack_hex_conv_weight")
            self._ops.append(op)
            return out.data_ptr()

        def lin_w(*weights: torch.Tensor) -> int:
            src = stage(*weights)
            n, k = src.shape
            out = torch.empty(n, _round_up(k, 64), dtype=torch.float16, device=device)
            self.keep.append(out)

            def op(src=src, out=out, n=n, k=k):
                _lib.check(_lib.lib().sb_pack_linear_weight(src.data_ptr(), n, k, out.data_ptr(),
                                                            torch.cuda.current_stream(device).cuda_stream),
                           "sb_pack_linear_weight")
            self._ops.append(op)
            return out.data_ptr()

        net.stem_w = conv_w(model.stem, 16)
        net.stem_b = f32(model.stem.bias)
        net.stem_ln_w = f32(model.stem_ln.weight)
        net.stem_ln_b = f32(model.stem_ln.bias)
        net.tokens = f32(model.tokens)
        # LN1 of the first attention block applied to the learned tokens (the
        # token rows of that block's input never pass through a conv)
        a0 = model.attn_blocks[0]
        tl16 = torch.empty(K.NUM_TOKENS, c, dtype=torch.float16, device=device)
        self.keep.append(tl16)
        self._ops.append(lambda: tl16.copy_(F.layer_norm(
            model.tokens.detach().to(device, torch.float32), (c,), a0.ln1.weight.detach().to(device, torch.float32),
            a0.ln1.bias.detach().to(device, torch.float32), a0.ln1.eps)))
        net.tokens_ln16 = tl16.data_ptr()
        net.ln_final_w = f32(model.ln_final.weight)
        net.ln_final_b = f32(model.ln_final.bias)
        net.policy_conv_w = conv_w(model.policy_conv, c)
        net.policy_conv_b = f32(model.policy_conv.bias)
        net.policy_head_w = f32(model.policy_head.weight.reshape(-1))
        net.policy_head_b = f32(model.policy_head.bias)
        net.value_red_wT = f32(model.value_reduction.weight.t())
        net.value_red_b = f32(model.value_reduction.bias)
        net.value_head_wT = f32(model.value_head.weight.t())
        net.value_head_b = f32(model.value_head.bias)
        net.ml_red_wT = f32(model.ml_reduction.weight.t())
        net.ml_red_b = f32(model.ml_reduction.bias)
        net.ml_head_wT = f32(model.moves_left_head.weight.t())
        net.ml_head_b = f32(model.moves_left_head.bias)
        lut = model._cell_bias_lut_u8
        if lut.device != device:
            lut = lut.to(device)
        self.keep.append(lut)
        net.lut = lut.data_ptr()
        for i, blk in enumerate(model.conv_blocks):
            cw = net.conv[i]
            cw.w1 = conv_w(blk.conv1, c)
            cw.b1 = f32(blk.conv1.bias)
            cw.ln1_w = f32(blk.ln1.weight)
            cw.ln1_b = f32(blk.ln1.bias)
            cw.w2 = conv_w(blk.conv2, c)
            cw.b2 = f32(blk.conv2.bias)
            cw.ln2_w = f32(blk.ln2.weight)
            cw.ln2_b = f32(blk.ln2.bias)
            cw.gamma = f32(blk.ls.gamma)
        for i, blk in enumerate(model.attn_blocks):
            aw = net.attn[i]
            at = blk.attn
            aw.ln1_w = f32(blk.ln1.weight)
            aw.ln1_b = f32(blk.ln1.bias)
            aw.wqkv = lin_w(at.q_proj.weight, at.k_proj.weight, at.v_proj.weight)
            qkv_b = stage(at.q_proj.bias, at.k_proj.bias, at.v_proj.bias)
            self.keep.append(qkv_b)
            aw.bqkv = qkv_b.data_ptr()
            aw.wo = lin_w(at.out_proj.weight)
            aw.bo = f32(at.out_proj.bias)
            aw.gamma_attn = f32(blk.ls_attn.gamma)
            aw.ln2_w = f32(blk.ln2.weight)
            aw.ln2_b = f32(blk.ln2.bias)
            aw.w1 = lin_w(blk.fc1.weight)
            aw.b1 = f32(blk.fc1.bias)
            aw.w2 = lin_w(blk.fc2.weight)
            aw.b2 = f32(blk.fc2.bias)
            aw.gamma_mlp = f32(blk.ls_mlp.gamma)
            # The reference adds the table rounded to fp16 (model.py:741); row
            # BIAS_ROWS is the additive pad-key row.
            tab = torch.empty(K.BIAS_ROWS + 1, h, dtype=torch.float32, device=device)
            self.keep.append(tab)

            def op(tab=tab, src=model.bias_tables[i]):
                tab[:K.BIAS_ROWS].copy_(src.detach().to(device).to(torch.float16))
                tab[K.BIAS_ROWS:].fill_(K.PAD_KEY_MASK_VALUE)
            self._ops.append(op)
            aw.bias_table = tab.data_ptr()
        self.net = net
        self.refresh()

    def refresh(self) -> None:
        """Re-pack the current parameter values into this object's buffers on
        the current stream (device work only)."""

        with torch.no_grad(), torch.autocast(device_type="cuda", enabled=False):
            for op in self._ops:
                op()
        self.packed_in_capture = torch.cuda.is_current_stream_capturing()


class ShrimpNet(nn.Module):
    """The Shrimp network (model.py:558-669): stem, trunk layout of ConvBlocks
    ('C') and AttnBlocks ('A'), ln_final, policy / value / auxiliary heads."""

    def __init__(
        self,
        channels: int = K.CHANNELS,
        attention_heads: int | None = None,
        trunk_layout: str | None = None,
    ) -> None:
        super().__init__()
        c = int(channels)
        heads = K.ATTENTION_HEADS if attention_heads is None else int(attention_heads)
        layout = K.validate_layout(K.TRUNK_LAYOUT if trunk_layout is None else str(trunk_layout))
        if c % heads:
            raise ValueError(f"channels={c} not divisible by attention_heads={heads}")
        self._trunk_layout = layout
        self.channels = c
        self.heads = heads
        self.stem = HexNodeConv(K.NUM_FEATURES, c)
        self.stem_ln = nn.LayerNorm(c)
        self.conv_blocks = nn.ModuleList([ConvBlock(c) for _ in range(layout.count("C"))])
        self.attn_blocks = nn.ModuleList([AttnBlock(c, heads) for _ in range(layout.count("A"))])
        self.tokens = nn.Parameter(torch.empty(K.NUM_TOKENS, c))
        self.bias_tables = nn.ParameterList(
            [nn.Parameter(torch.zeros(K.BIAS_ROWS, heads)) for _ in range(len(self.attn_blocks))]
        )
        self.ln_final = nn.LayerNorm(c)
        self.policy_conv = HexNodeConv(c, c)
        self.policy_head = nn.Linear(c, 1)
        self.opp_policy_conv = HexNodeConv(c, c)
        self.opp_policy_head = nn.Linear(c, 1)
        self.soft_policy_conv = HexNodeConv(c, c)
        self.soft_policy_head = nn.Linear(c, 1)
        self.cell_q_conv = HexNodeConv(c, c)
        self.cell_q_head = nn.Linear(c, K.VALUE_BINS)
        self.value_reduction = nn.Linear(3 * c, c)
        self.value_head = nn.Linear(c, K.VALUE_BINS)
        self.aux_reduction = nn.Linear(3 * c, c)
        self.stv_heads = nn.ModuleDict({str(hz): nn.Linear(c, K.VALUE_BINS) for hz in STV_HORIZONS})
        self.ml_reduction = nn.Linear(3 * c, c)
        self.moves_left_head = nn.Linear(c, K.VALUE_BINS)
        self.register_buffer(
            "_cell_bias_lut_u8", torch.from_numpy(cell_bias_lut().copy()), persistent=False
        )
        self._init_weights()
        self._packed: dict = {}
        self._param_list = None
        self._workspace: dict = {}
        self._retired_workspaces: list = []
        # load_state_dict(assign=True) replaces parameter objects: re-read the
        # parameter list (an in-place load keeps the packed buffers, which are
        # re-packed in place, so graphs captured before it stay valid)
        self.register_load_state_dict_post_hook(lambda module, keys: setattr(module, "_param_list", None))

    def _init_weights(self) -> None:
        """Linear: trunc_normal(0.02) weight, zero bias; LayerNorm: (1, 0);
        tokens: trunc_normal(0.02); convs, gammas and tables keep their own
        init (model.py:655-669)."""

        for module in self.modules():
            if isinstance(module, nn.Linear):
                nn.init.trunc_normal_(module.weight, std=0.02)
                nn.init.zeros_(module.bias)
            elif isinstance(module, nn.LayerNorm):
                nn.init.ones_(module.weight)
                nn.init.zeros_(module.bias)
        nn.init.trunc_normal_(self.tokens, std=0.02)

    def set_attention_impl(self, impl: str) -> None:
        """Accepted for API compatibility (model.py:671-673); the native
        attention kernel is the only implementation."""

        if impl not in ("sdpa", "materialized"):
            raise ValueError(f"unknown attention impl: {impl}")
        for block in self.attn_blocks:
            block.attn.impl = impl

    # --- native serve path -------------------------------------------------------

    def _apply(self, fn, *args, **kwargs):
        # .to() / .half() / .cuda() swap parameter storage: build new buffers
        out = super()._apply(fn, *args, **kwargs)
        self.invalidate_packed()
        return out

    def invalidate_packed(self) -> None:
        """Drop the packed weights; the next forward builds them again. Needed
        only after replacing parameter objects by hand (assigning a new
        nn.Parameter): in-place updates, load_state_dict and module
        conversions are detected on their own. Like a module conversion
        (.to / .half), this frees buffers that CUDA graphs captured before it
        point to: capture those graphs again."""

        self._packed = {}
        self._param_list = None

    def _weights_state(self) -> list:
        if self._param_list is None:
            self._param_list = list(self.parameters())
        return [(p.data_ptr(), p._version) for p in self._param_list]

    def packed(self, device: torch.device) -> PackedWeights:
        """The packed weights for `device`, brought up to date: rebuilt when a
        parameter's storage changed, re-packed in place when only its values
        changed (in-place update, load_state_dict), and re-packed eagerly once
        after a pack that was recorded inside a CUDA-graph capture (recorded
        work runs only when the graph replays)."""

        state = self._weights_state()
        entry = self._packed.get(device)
        capturing = torch.cuda.is_current_stream_capturing()
        if entry is None or [p for p, _ in entry[1]] != [p for p, _ in state]:
            entry = (PackedWeights(self, device), state)
            self._packed[device] = entry
        elif entry[1] != state or (entry[0].packed_in_capture and not capturing):
            entry[0].refresh()
            entry = (entry[0], state)
            self._packed[device] = entry
        return entry[0]

    def _workspace_for(self, device: torch.device, batch: int, npad: int) -> torch.Tensor:
        net = self.packed(device).net
        nbytes = C.c_size_t(0)
        _lib.check(_lib.lib().sb_forward_workspace_bytes(C.byref(net), batch, npad, C.byref(nbytes)),
                   "sb_forward_workspace_bytes")
        ws = self._workspace.get(device)
        if ws is None or ws.numel() < nbytes.value:
            # A CUDA graph captured with the old workspace keeps its address, so
            # the old one stays allocated (retired); growing by at least 1.5x
            # bounds the retired bytes by twice the final size.
            if ws is not None:
                self._retired_workspaces.append(ws)
            size = max(nbytes.value, 1 if ws is None else int(ws.numel() * 1.5))
            ws = torch.empty(size, dtype=torch.uint8, device=device)
            self._workspace[device] = ws
        return ws

    @torch.compiler.disable
    @torch.no_grad()
    def forward_policy_value(
        self,
        feats: torch.Tensor,
        nbr: torch.Tensor,
        mask: torch.Tensor,
        coords: torch.Tensor,
        *,
        request_moves_left: bool = False,
        out: dict | None = None,
        status: torch.Tensor | None = None,
    ) -> dict[str, torch.Tensor]:
        """Serve forward (model.py:972-1003): {'policy' (B, Npad) fp32 logits with
        pad rows 0, 'value' (B, 65) fp32 bin logits[, 'moves_left' (B, 65)]}.

        Inputs: feats (B, Npad, 15) f32/f16/bf16, nbr (B, Npad, 6) int64/int32
        (missing = Npad), mask (B, Npad) bool, coords (B, Npad, 2) int64/int32,
        all on one CUDA device. `out` may supply preallocated output tensors
        (keys policy, value[, moves_left]) for CUDA-graph capture."""

        for name, t in (("feats", feats), ("nbr", nbr), ("mask", mask), ("coords", coords)):
            if not t.is_cuda:
                raise RuntimeError(
                    f"ShrimpNet.forward_policy_value: {name} is on {t.device}; the B200 build runs "
                    "only on CUDA tensors (no CPU fallback)"
                )
        device = feats.device
        b, npad = int(feats.shape[0]), int(feats.shape[1])
        if feats.shape[2] != K.NUM_FEATURES or nbr.shape != (b, npad, 6) or mask.shape != (b, npad) or \
                coords.shape != (b, npad, 2):
            raise ValueError("forward_policy_value: inconsistent input shapes")
        feats = feats.contiguous()
        nbr = nbr.contiguous()
        mask = mask.contiguous()
        coords = coords.contiguous()
        if out is None:
            out = {
                "policy": torch.empty(b, npad, dtype=torch.float32, device=device),
                "value": torch.empty(b, K.VALUE_BINS, dtype=torch.float32, device=device),
            }
            if request_moves_left:
                out["moves_left"] = torch.empty(b, K.VALUE_BINS, dtype=torch.float32, device=device)
        if b == 0:
            return out
        pk = self.packed(device)
        ws = self._workspace_for(device, b, npad)
        ins = _lib.Inputs(
            feats.data_ptr(), _dtype_code(feats), nbr.data_ptr(), _dtype_code(nbr),
            mask.data_ptr(), _dtype_code(mask), coords.data_ptr(), _dtype_code(coords), b, npad,
        )
        outs = _lib.Outputs(
            out["policy"].data_ptr(), out["value"].data_ptr(), None,
            _ptr(out.get("moves_left")) if request_moves_left else None, None,
            _ptr(status),
        )
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(
            _lib.lib().sb_forward_policy_value(C.byref(pk.net), C.byref(ins), C.byref(outs), ws.data_ptr(),
                                               ws.numel(), stream),
            "sb_forward_policy_value",
        )
        return out

    def forward(self, *args, **kwargs):
        raise NotImplementedError(
            "ShrimpNet.forward (training heads) is not part of the B200 serve build; "
            "use forward_policy_value"
        )

    @staticmethod
    def kernel_launches(layout: str, grid: bool = False, channels: int = 128, pooled: bool = False) -> int:
        """Kernels one forward_policy_value call enqueues. With `grid` (dense
        inputs of at most 81 cells, channels a multiple of 64 up to 128, at
        least 1024 positions) the geometry check runs and the first conv of
        every ConvBlock and the policy conv are launched twice, as the grid
        conv and as the windowed conv, one of which returns at once. An
        attention block is four launches (qkv, core, out_proj, the fused MLP)
        at 64 or 128 channels and five (fc1 and fc2 apart) otherwise. With
        `pooled` (see pools_cells_apart) the cell mean of the value heads is
        one more launch."""

        n_conv = layout.count("C")
        dual = n_conv + 1 if grid else 0
        per_attn = 4 if channels in (64, 128) else 5
        return (2 + (1 if grid else 0) + 1 + 2 * n_conv + 1 + dual + per_attn * layout.count("A") + 1
                + (1 if pooled else 0))

    @staticmethod
    def pools_cells_apart(batch: int, npad: int, sms: int = 148) -> bool:
        """The native rule for pooling the heads' cell mean in a kernel of its
        own: fewer heads CTAs (four positions each) than SMs, and more than
        one 128-row chunk of cells per position."""

        return (batch + 3) // 4 < sms and (npad + 127) // 128 > 1


__all__ = ["ShrimpNet", "HexNodeConv", "ConvBlock", "AttnBlock", "RelPosAttention", "LayerScale",
           "PackedWeights", "infer_net_kwargs_from_state_dict", "KNOWN_TRUNK_LAYOUTS"]
