"""Block-scaled FP8 quantizer and tcgen05 kind::mxf8f6f4 GEMM (csrc/gemm_mx.cu)
against plain PyTorch: the quantizer bit for bit against its torch
restatement, the GEMM against an fp32 matmul of the dequantized operands."""
import pytest

pytestmark = pytest.mark.gpu


def _rel(a, b):
    import torch
    return (torch.linalg.vector_norm(a.float() - b.float()) / torch.linalg.vector_norm(b.float()).clamp_min(1e-30)).item()


def test_quantizer_matches_reference(cuda):
    import torch
    from tempname_dcu_b200.ops import mx, native
    torch.manual_seed(0)
    x = (torch.randn(256, 512) * torch.logspace(-4, 4, 512)).to(torch.bfloat16)
    x[:, 64:96] = 0  # an all-zero block
    xd = x.to(cuda)
    q, sf = mx.quantize(xd)
    torch.cuda.synchronize()
    values, e = mx.quantize_reference(x)
    assert torch.equal(mx.scales_dense(sf.cpu(), 256, 512).long(), (e + 127).long())
    assert torch.equal(q.cpu().view(torch.float8_e4m3fn).float(), values)
    assert native.read_status()[0] == 0


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 384, 512), (1024, 1536, 2048), (2048, 4096, 4096)])
def test_mx_gemm_matches_dequantized_fp32(cuda, M, N, K):
    import torch
    from tempname_dcu_b200.ops import mx, native
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) * 0.02).to(torch.bfloat16)
    qa, sfa = mx.quantize(x)
    qb, sfb = mx.quantize(w)
    y = mx.gemm(qa, sfa, qb, sfb)
    ref = mx.dequantize(qa, sfa) @ mx.dequantize(qb, sfb).t()
    assert _rel(y, ref) < 5e-3
    # and the quantization error against the bf16 product stays at the e4m3 level
    assert _rel(y, x.float() @ w.float().t()) < 6e-2
    assert native.read_status()[0] == 0


def test_mx_gemm_bias_and_strided_output(cuda):
    import torch
    from tempname_dcu_b200.ops import mx
    torch.manual_seed(3)
    x = torch.randn(512, 256, device=cuda).to(torch.bfloat16)
    w = torch.randn(384, 256, device=cuda).to(torch.bfloat16)
    b = torch.randn(384, device=cuda).to(torch.bfloat16)
    qa, sfa = mx.quantize(x)
    qb, sfb = mx.quantize(w)
    big = torch.zeros(512, 512, device=cuda, dtype=torch.bfloat16)
    out = big[:, :384]
    mx.gemm(qa, sfa, qb, sfb, bias=b, out=out)
    ref = mx.dequantize(qa, sfa) @ mx.dequantize(qb, sfb).t() + b.float()
    assert _rel(out, ref) < 5e-3
    assert big[:, 384:].abs().max().item() == 0


def test_versioned_quantization_skips_until_the_version_moves(cuda):
    import torch
    from tempname_dcu_b200.ops import mx
    x = torch.randn(256, 256, device=cuda).to(torch.bfloat16)
    version = torch.zeros((), dtype=torch.int32, device=cuda)
    seen = torch.full((), -1, dtype=torch.int32, device=cuda)
    q, sf = mx.quantize(x, version=version, seen=seen)
    first = q.clone()
    assert seen.item() == 0
    x2 = (x * 3).to(torch.bfloat16)
    mx.quantize(x2, q, sf, version=version, seen=seen)  # same version: skipped on the device
    assert torch.equal(q, first)
    version.add_(1)
    mx.quantize(x2, q, sf, version=version, seen=seen)
    assert seen.item() == 1 and torch.equal(q, mx.quantize(x2)[0])
