"""sb_hex_conv_noalloc: the hex_conv entry point whose scratch is a fixed
device array inside the library. Compared with sb_hex_conv (caller
workspace) on two calls in a row; the size limit is checked without a GPU."""

import ctypes as C
import math

import pytest
import torch

from hexo_bot_b200 import _lib

TOL = 1e-3  # same kernels on the same inputs: expected bit-identical


def test_noalloc_rejects_batches_beyond_the_fixed_scratch():
    lib = _lib.lib()
    dummy = C.c_void_p(16)
    rc = lib.sb_hex_conv_noalloc(dummy, dummy, dummy, dummy, dummy, 4096, 64, 128, 128, dummy, None)
    assert rc == _lib.SB_ERR_UNSUPPORTED
    assert "262141" in _lib.last_error()
    # one row past the documented limit is refused before any device work
    rc = lib.sb_hex_conv_noalloc(dummy, dummy, dummy, dummy, dummy, 1, 262142, 128, 128, dummy, None)
    assert rc == _lib.SB_ERR_UNSUPPORTED


def _case(dev, b, n, cin, cout, seed):
    torch.manual_seed(seed)
    x = torch.randn(b, n, cin, device=dev).half()
    nbr = torch.randint(0, n + 1, (b, n, 6), device=dev)
    gidx = torch.cat([torch.arange(n, device=dev).view(1, n, 1).expand(b, -1, -1), nbr], 2).int().contiguous()
    mask = (torch.rand(b, n, device=dev) > 0.1).to(torch.uint8)
    w = torch.randn(7, cin, cout, device=dev) / math.sqrt(7 * cin)
    bias = torch.randn(cout, device=dev) * 0.1
    return x, gidx, mask, w, bias


def _workspace_result(lib, st, dev, x, gidx, mask, wp, bias, b, n, cin, cout):
    ref = torch.empty(b, n, cout, dtype=torch.float16, device=dev)
    nb = C.c_size_t()
    lib.sb_hex_conv_workspace_bytes(b, n, C.byref(nb))
    ws = torch.empty(nb.value, dtype=torch.uint8, device=dev)
    _lib.check(lib.sb_hex_conv(x.data_ptr(), gidx.data_ptr(), mask.data_ptr(), wp.data_ptr(), bias.data_ptr(), b, n,
                               cin, cout, ref.data_ptr(), ws.data_ptr(), nb.value, st), "hex_conv")
    return ref


@pytest.mark.gpu
def test_noalloc_larger_call_then_smaller_call():
    """A smaller call after a larger one reads none of the larger call's
    leftover gather rows or row mask from the shared scratch."""
    dev = torch.device("cuda")
    lib = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    for b, n, seed in ((64, 61, 21), (9, 40, 22)):
        cin = cout = 64
        x, gidx, mask, w, bias = _case(dev, b, n, cin, cout, seed)
        kpad = (7 * cin + 63) // 64 * 64
        wp = torch.empty(cout, kpad, dtype=torch.float16, device=dev)
        _lib.check(lib.sb_pack_hex_conv_weight(w.data_ptr(), 7, cin, cin, cout, wp.data_ptr(), st), "pack")
        ref = _workspace_result(lib, st, dev, x, gidx, mask, wp, bias, b, n, cin, cout)
        out = torch.full_like(ref, float("nan"))
        _lib.check(lib.sb_hex_conv_noalloc(x.data_ptr(), gidx.data_ptr(), mask.data_ptr(), wp.data_ptr(),
                                           bias.data_ptr(), b, n, cin, cout, out.data_ptr(), st), "hex_conv_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert (out.float() - ref.float()).abs().max().item() <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("b,n,cin,cout", [(64, 61, 128, 128), (9, 40, 32, 32)])
def test_noalloc_matches_workspace_entry_on_two_calls(b, n, cin, cout):
    dev = torch.device("cuda")
    lib = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    torch.manual_seed(7)
    x = torch.randn(b, n, cin, device=dev).half()
    nbr = torch.randint(0, n + 1, (b, n, 6), device=dev)
    gidx = torch.cat([torch.arange(n, device=dev).view(1, n, 1).expand(b, -1, -1), nbr], 2).int().contiguous()
    mask = (torch.rand(b, n, device=dev) > 0.1).to(torch.uint8)
    w = torch.randn(7, cin, cout, device=dev) / math.sqrt(7 * cin)
    bias = torch.randn(cout, device=dev) * 0.1
    kpad = (7 * cin + 63) // 64 * 64
    wp = torch.empty(cout, kpad, dtype=torch.float16, device=dev)
    _lib.check(lib.sb_pack_hex_conv_weight(w.data_ptr(), 7, cin, cin, cout, wp.data_ptr(), st), "pack")

    ref = torch.empty(b, n, cout, dtype=torch.float16, device=dev)
    nb = C.c_size_t()
    lib.sb_hex_conv_workspace_bytes(b, n, C.byref(nb))
    ws = torch.empty(nb.value, dtype=torch.uint8, device=dev)
    _lib.check(lib.sb_hex_conv(x.data_ptr(), gidx.data_ptr(), mask.data_ptr(), wp.data_ptr(), bias.data_ptr(), b, n,
                               cin, cout, ref.data_ptr(), ws.data_ptr(), nb.value, st), "hex_conv")
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        _lib.check(lib.sb_hex_conv_noalloc(x.data_ptr(), gidx.data_ptr(), mask.data_ptr(), wp.data_ptr(),
                                           bias.data_ptr(), b, n, cin, cout, out.data_ptr(), st), "hex_conv_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert (out.float() - ref.float()).abs().max().item() <= TOL
