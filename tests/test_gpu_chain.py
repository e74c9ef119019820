"""GPU: chained activations (bq4_linear_ex) and the layer-stack renorm.

A linear that writes its output as f16 rounds it exactly as the next
linear's staging would, and a linear that reads f16 activations in place
skips only that staging copy -- so a chain of linears must give the same
bits either way.  Also: outputs written into column slices of a wider
buffer, the per-token RMS renorm against torch, the chained DiT stack
against the float32 stack, and the argument checks of the new entry points.
"""
import pytest
import torch

from burn_image_b200 import _lib as L
from burn_image_b200 import q4, tp
from burn_image_b200.q4 import Bq4Error

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _weight(K, N, g, block=128):
    w, s = tp._random_packed(K, N, block, g, DEV)
    return q4.PreparedQ4Weight(w, s, K, N, block, L.LAYOUT_ROW, DEV)


# exact (M <= 64), folded with operand A in TMEM (large M), and a split-K plan
@pytest.mark.parametrize("M,K,N", [(48, 512, 640), (4352, 1024, 2048), (256, 2560, 2560)])
def test_f16_chain_is_bit_identical(M, K, N):
    g = torch.Generator(device=DEV).manual_seed(M + K)
    w1, w2 = _weight(K, N, g), _weight(N, K, g)
    bias = torch.randn(N, generator=g, device=DEV) * 0.02
    x = torch.randn((M, K), generator=g, device=DEV)
    y32 = w1.linear(x, bias, L.ACT_GELU_TANH)
    y16 = w1.linear_ex(x, bias, L.ACT_GELU_TANH, out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(y16, y32.half())
    z32 = w2.linear(y32)
    z16in = w2.linear_ex(y16)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(z16in, z32)


def test_outputs_into_column_slices():
    M, K, N = 300, 1024, 384
    g = torch.Generator(device=DEV).manual_seed(5)
    w = _weight(K, N, g)
    x = torch.randn((M, K), generator=g, device=DEV)
    ref = w.linear(x)
    for dtype in (torch.float32, torch.float16):
        wide = torch.full((M, 3 * N), 7.0, dtype=dtype, device=DEV)
        w.linear_ex(x, out=wide[:, N:2 * N])
        torch.cuda.synchronize()
        assert torch.equal(wide[:, N:2 * N], ref.to(dtype))
        assert (wide[:, :N] == 7.0).all() and (wide[:, 2 * N:] == 7.0).all()
    # f16 input read from a column slice (row pitch > K)
    xs = torch.zeros((M, K + 128), dtype=torch.float16, device=DEV)
    xs[:, 128:] = x.half()
    assert torch.equal(w.linear_ex(xs[:, 128:]), ref)


def test_rms_renorm_matches_torch():
    g = torch.Generator(device=DEV).manual_seed(9)
    d = torch.randn((517, 3072), generator=g, device=DEV) * 3.0
    ref = d.double() * torch.rsqrt(d.double().pow(2).mean(-1, keepdim=True) + 1e-6)
    out32 = q4.rms_renorm(d, torch.empty_like(d))
    out16 = q4.rms_renorm(d, torch.empty_like(d, dtype=torch.float16))
    in16 = q4.rms_renorm(d.half(), torch.empty_like(d))
    torch.cuda.synchronize()
    assert (out32.double() - ref).abs().max().item() < 1e-5
    assert (out16.double() - ref).abs().max().item() < 2e-3  # one f16 rounding of |v| < 8
    ref16 = d.half().double() * torch.rsqrt(d.half().double().pow(2).mean(-1, keepdim=True) + 1e-6)
    assert (in16.double() - ref16).abs().max().item() < 1e-5
    # an unaligned column slice (width 3071) takes the scalar kernel
    ds = d[:, 1:]
    refs = ds.double() * torch.rsqrt(ds.double().pow(2).mean(-1, keepdim=True) + 1e-6)
    outs = q4.rms_renorm(ds, torch.empty((517, 3071), device=DEV))
    torch.cuda.synchronize()
    assert (outs.double() - refs).abs().max().item() < 1e-5


def test_chained_stack_matches_float32_stack():
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn((300, 512), generator=g, device=DEV)
    s32 = tp.DiTQ4Stack(2, 512, 1536, 2048, DEV, seed=4)
    s16 = tp.DiTQ4Stack(2, 512, 1536, 2048, DEV, seed=4, act_dtype=torch.float16, chunks=2)
    a, b = s32.forward(x), s16.forward(x)
    torch.cuda.synchronize()
    q4.poll_device_error()
    rel = (torch.linalg.norm(a.double() - b.double()) / torch.linalg.norm(a.double())).item()
    assert rel < 1e-3  # the two renorm kernels round differently; the linears agree bit for bit


def test_linear_ex_argument_checks():
    g = torch.Generator(device=DEV).manual_seed(1)
    w = _weight(576, 256, g, block=64)  # K = 576 is not a multiple of 128: f16 input cannot be read in place
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        w.linear_ex(torch.zeros((8, 576), dtype=torch.float16, device=DEV))
    w2 = _weight(512, 256, g)
    x = torch.zeros((8, 520), dtype=torch.float16, device=DEV)
    with pytest.raises(Bq4Error, match="EALIGN"):
        w2.linear_ex(x[:, 4:516])  # base not 16-byte aligned
    with pytest.raises(Bq4Error):
        w2.linear_ex(torch.zeros((8, 512), dtype=torch.float16, device=DEV),
                     out=torch.empty((8, 255), device=DEV))
