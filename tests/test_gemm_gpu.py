"""tcgen05 GEMM (csrc/gemm.cu) against a plain fp32 PyTorch reference."""
import pytest

pytestmark = pytest.mark.gpu


def _rel(a, b):
    import torch
    return (torch.linalg.vector_norm(a.float() - b.float()) / torch.linalg.vector_norm(b.float()).clamp_min(1e-30)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (300, 264, 200), (1024, 1536, 512),
                                   (2048, 4096, 1024)])
def test_linear_kk(cuda, M, N, K):
    import torch
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(0)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = torch.randn(N, K, device=cuda).to(torch.bfloat16)
    y = g.linear(x, w)
    ref = x.float() @ w.float().t()
    assert _rel(y, ref) < 5e-3
    g_status = __import__("tempname_dcu_b200.ops.native", fromlist=["x"]).read_status()
    assert g_status[0] == 0


@pytest.mark.parametrize("bn", [128, 192, 256])
def test_both_tile_widths(cuda, bn):
    import torch
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(1)
    x = torch.randn(512, 256, device=cuda).to(torch.bfloat16)
    w = torch.randn(768, 256, device=cuda).to(torch.bfloat16)
    y = g.gemm(x, w, bn=bn)
    assert _rel(y, x.float() @ w.float().t()) < 5e-3


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (384, 640, 192), (2048, 1024, 512)])
def test_data_gradient_b_mn_major(cuda, M, N, K):
    import torch
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(2)
    dy = torch.randn(M, N, device=cuda).to(torch.bfloat16)
    w = torch.randn(N, K, device=cuda).to(torch.bfloat16)
    dx = g.matmul_nt(dy, w)
    assert _rel(dx, dy.float() @ w.float()) < 5e-3


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (512, 384, 320), (2048, 512, 768)])
def test_weight_gradient_mn_mn_accumulate(cuda, M, N, K):
    import torch
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(3)
    dy = torch.randn(M, N, device=cuda).to(torch.bfloat16)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    acc = torch.randn(N, K, device=cuda)
    base = acc.clone()
    g.weight_grad(dy, x, acc, accumulate=True)
    ref = base + dy.float().t() @ x.float()
    assert _rel(acc, ref) < 2e-3
    fresh = g.weight_grad(dy, x)
    assert _rel(fresh, dy.float().t() @ x.float()) < 2e-3


def test_fused_epilogues(cuda):
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(4)
    M, N, K = 384, 512, 256
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) / 16).to(torch.bfloat16)
    b = torch.randn(N, device=cuda).to(torch.bfloat16)
    res = torch.randn(M, N, device=cuda).to(torch.bfloat16)
    z_ref = x.float() @ w.float().t() + b.float()
    y = g.linear(x, w, b)
    assert _rel(y, z_ref) < 5e-3
    act, pre = g.linear_gelu(x, w, b)
    assert _rel(pre, z_ref) < 5e-3
    assert _rel(act, F.gelu(pre.float())) < 5e-3
    out = g.linear_residual(x, w, b, res)
    assert _rel(out, z_ref + res.float()) < 5e-3
    # GELU backward: dz = (dy @ w2) * gelu'(pre)
    dy = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w2 = (torch.randn(K, N, device=cuda) / 16).to(torch.bfloat16)
    dz = g.matmul_nt(dy, w2, gelu_pre=pre)
    pre_f = pre.float().requires_grad_(True)
    F.gelu(pre_f).backward((dy.float() @ w2.float()))
    assert _rel(dz, pre_f.grad) < 1e-2


def test_large_k_and_many_tiles(cuda):
    import torch
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(5)
    x = torch.randn(1024, 4096, device=cuda).to(torch.bfloat16)
    w = torch.randn(4096, 4096, device=cuda).to(torch.bfloat16)
    y = g.linear(x, w)
    assert _rel(y, x.float() @ w.float().t()) < 5e-3


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 320), (600, 520, 200), (2048, 4096, 1024)])
def test_two_cta_tiles_all_layouts(cuda, a_mn, b_mn, M, N, K):
    """cta_group::2 (SM-pair) 256x256 tiles, requested with bn=512."""
    import torch
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(6)
    A = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    B = torch.randn(N, K, device=cuda).to(torch.bfloat16)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    if a_mn:
        out = g.gemm(a, b, a_mn=True, b_mn=b_mn, mode=g.ACC_F32, bn=512)
        assert _rel(out, ref) < 2e-3
    else:
        out = g.gemm(a, b, a_mn=a_mn, b_mn=b_mn, bn=512)
        assert _rel(out, ref) < 5e-3
    from tempname_dcu_b200.ops import native
    assert native.read_status()[0] == 0


def test_two_cta_fused_epilogues(cuda):
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(7)
    M, N, K = 512, 1024, 512
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) / 16).to(torch.bfloat16)
    b = torch.randn(N, device=cuda).to(torch.bfloat16)
    res = torch.randn(M, N, device=cuda).to(torch.bfloat16)
    z_ref = x.float() @ w.float().t() + b.float()
    pre = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    act = g.gemm(x, w, mode=g.BIAS_GELU, bias=b, aux_out=pre, bn=512)
    assert _rel(pre, z_ref) < 5e-3 and _rel(act, F.gelu(pre.float())) < 5e-3
    out = g.gemm(x, w, mode=g.BIAS_RESIDUAL, bias=b, aux=res, bn=512)
    assert _rel(out, z_ref + res.float()) < 5e-3


@pytest.mark.parametrize("a_mn,b_mn,mode", [(False, False, "bias_gelu"), (False, True, "store"), (True, True, "acc")])
def test_192_wide_tiles_ragged(cuda, a_mn, b_mn, mode):
    """128 x 192 tiles with N not a multiple of 192 (TP-sized shapes)."""
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import gemm as g
    torch.manual_seed(9)
    M, N, K = 512, 1000, 384
    A = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    B = (torch.randn(N, K, device=cuda) / 8).to(torch.bfloat16)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    if mode == "acc":
        acc = torch.randn(M, N, device=cuda)
        base = acc.clone()
        g.gemm(a, b, a_mn=a_mn, b_mn=b_mn, out=acc, mode=g.ACC_F32, beta=1.0, bn=192)
        assert _rel(acc, base + ref) < 2e-3
    elif mode == "bias_gelu":
        bias = torch.randn(N, device=cuda).to(torch.bfloat16)
        pre = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
        act = g.gemm(a, b, mode=g.BIAS_GELU, bias=bias, aux_out=pre, bn=192)
        assert _rel(pre, ref + bias.float()) < 5e-3 and _rel(act, F.gelu(pre.float())) < 5e-3
    else:
        out = g.gemm(a, b, a_mn=a_mn, b_mn=b_mn, bn=192)
        assert _rel(out, ref) < 5e-3
