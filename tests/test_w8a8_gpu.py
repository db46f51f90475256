"""GPU parity for the W8A8 path through the C ABI: quantisation, int32 accumulators and the bf16 epilogue are
all bit-exact against the CPU oracle (oracle/w8a8.py). Shapes with K >= 8192 and M >= 1024 run the CTA-pair
kernel (ragged M, N and K included); the others the one-CTA kernel. Each shape also runs without the int32
accumulator copy and without bias."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from gpu_util import bf16_cuda, bits_np
from oracle import w8a8 as ow

pytestmark = pytest.mark.gpu


def test_w8a8_golden_bit_exact(cuda_lib):
    from hummingbird_b200.w8a8 import quantize_rows, w8a8_gemm
    z = load_golden("w8a8_m9_k96_n12")
    # pad N to a multiple of 32 (kernel requirement) with zero weight rows; compare the first 12 columns
    x = bf16_cuda(z["x_bits"])
    w = np.zeros((32, 96), np.uint16)
    w[:12] = z["w_bits"]
    qx, sx = quantize_rows(x)
    qw, sw = quantize_rows(bf16_cuda(w))
    bias = np.zeros(32, np.uint16)
    bias[:12] = z["bias_bits"]
    acc = torch.empty(9, 32, dtype=torch.int32, device="cuda")
    y = w8a8_gemm(qx, sx, qw, sw, bf16_cuda(bias), acc_out=acc)
    torch.cuda.synchronize()
    assert np.array_equal(qx.cpu().numpy(), z["qx"])
    assert np.array_equal(sx.cpu().numpy(), z["sx"])
    assert np.array_equal(qw.cpu().numpy()[:12], z["qw"])
    assert np.array_equal(acc.cpu().numpy()[:, :12], z["acc"])
    assert np.array_equal(bits_np(y)[:, :12], z["y_bits"])


@pytest.mark.parametrize("m,k,n", [(2584, 1024, 4096), (2584, 4096, 1024), (1100, 8192, 1024), (1030, 8208, 352),
                                   (1300, 512, 1024), (513, 272, 96), (200, 272, 96), (1, 16, 32), (300, 384, 320),
                                   (1, 128, 64), (5296, 1024, 5120)])
def test_w8a8_gemm_bit_exact(m, k, n, cuda_lib):
    from hummingbird_b200.w8a8 import quantize_rows, w8a8_gemm
    g = torch.Generator(device="cuda").manual_seed(m * 7 + k * 3 + n)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
    bias = (0.02 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    qx, sx = quantize_rows(x)
    qw, sw = quantize_rows(w)
    acc = torch.empty(m, n, dtype=torch.int32, device="cuda")
    y = w8a8_gemm(qx, sx, qw, sw, bias, acc_out=acc)
    torch.cuda.synchronize()
    xq_ref, sx_ref = ow.quantize_rows(x.float().cpu().numpy())
    wq_ref, sw_ref = ow.quantize_rows(w.float().cpu().numpy())
    assert np.array_equal(qx.cpu().numpy(), xq_ref) and np.array_equal(sx.cpu().numpy(), sx_ref)
    assert np.array_equal(qw.cpu().numpy(), wq_ref) and np.array_equal(sw.cpu().numpy(), sw_ref)
    acc_ref = ow.int_matmul(xq_ref, wq_ref)
    assert np.array_equal(acc.cpu().numpy(), acc_ref)
    y_ref = ow.epilogue(acc_ref, sx_ref, sw_ref, bits_np(bias))
    assert np.array_equal(bits_np(y), y_ref)
    # without the accumulator copy, and without bias
    y2 = w8a8_gemm(qx, sx, qw, sw, bias)
    y3 = w8a8_gemm(qx, sx, qw, sw, None)
    torch.cuda.synchronize()
    assert np.array_equal(bits_np(y2), y_ref)
    assert np.array_equal(bits_np(y3), ow.epilogue(acc_ref, sx_ref, sw_ref, None))


def test_w8a8_linear_pair_config3(cuda_lib):
    """Config 3: GEMM1 (1024 -> 4096) then GEMM2 (4096 -> 1024) on GEMM1's bf16 output, bit-exact."""
    from hummingbird_b200.w8a8 import W8A8Linear
    from hummingbird_b200.workloads import w8a8_inputs
    w = w8a8_inputs("cuda")
    l1, l2 = W8A8Linear(w.w1, w.b1), W8A8Linear(w.w2, w.b2)
    h = l1(w.x)
    y = l2(h)
    torch.cuda.synchronize()
    h_ref, _, _, _ = ow.w8a8_linear(bits_np(w.x), l1.qw.cpu().numpy(), l1.sw.cpu().numpy(), bits_np(w.b1))
    assert np.array_equal(bits_np(h), h_ref)
    y_ref, _, _, _ = ow.w8a8_linear(h_ref, l2.qw.cpu().numpy(), l2.sw.cpu().numpy(), bits_np(w.b2))
    assert np.array_equal(bits_np(y), y_ref)


@pytest.mark.parametrize("m,k,f", [(2584, 1024, 4096), (5296, 1024, 4096), (200, 96, 256), (129, 1040, 384)])
def test_w8a8_gemm_glu_epilogue_bit_exact(cuda_lib, m, k, f):
    """The GEMM with the GLU in its epilogue (`hb_w8a8_gemm_glu`, weight rows in `glu_interleave` order) against
    the unfused sequence it replaces: the plain GEMM's bf16 output, then `hb_glu_rows`. z is bit-identical, and so
    is its per-row int8 form (`hb_quant_rows_int8` on the fused z against `hb_glu_rows`' int8 mode). Ragged M,
    K past whole 128-byte stages, and F of one to 32 value/gate tile pairs."""
    from hummingbird_b200 import _lib, dit_glue
    from hummingbird_b200.w8a8 import W8A8GluLinear, glu_interleave, quantize_rows, w8a8_gemm
    g = torch.Generator(device="cuda").manual_seed(m + k + f)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(2 * f, k, generator=g, device="cuda") / k ** 0.5).to(torch.bfloat16)
    bias = (0.05 * torch.randn(2 * f, generator=g, device="cuda")).to(torch.bfloat16)
    qx, sx = quantize_rows(x)
    qw, sw = quantize_rows(w)
    plain = w8a8_gemm(qx, sx, qw, sw, bias)
    z_ref = dit_glue.glu(plain)
    q_ref, s_ref = dit_glue.glu(plain, quantize=True)
    lin = W8A8GluLinear(w, bias)
    assert torch.equal(lin.qw, glu_interleave(qw)) and torch.equal(lin.sw, glu_interleave(sw))
    z = lin(x)
    q, s = quantize_rows(z)
    torch.cuda.synchronize()
    assert np.array_equal(bits_np(z), bits_np(z_ref))
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)
    assert _lib.device_status() == 0
