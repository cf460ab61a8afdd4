"""LayerNorm, attention, cross-entropy, AdamW, grad-norm and embedding kernels
against plain fp32 PyTorch references of the same ops."""
import math

import pytest

pytestmark = pytest.mark.gpu


def _rel(a, b):
    import torch
    return (torch.linalg.vector_norm(a.float() - b.float()) / torch.linalg.vector_norm(b.float()).clamp_min(1e-30)).item()


@pytest.mark.parametrize("rows,H", [(64, 4096), (37, 256), (16, 1024)])
def test_layernorm_fwd_bwd(cuda, rows, H):
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(0)
    x = (torch.randn(rows, H, device=cuda) * 3 + 1).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device=cuda)).to(torch.bfloat16)
    b = (0.1 * torch.randn(H, device=cuda)).to(torch.bfloat16)
    y, mean, rstd = k.layernorm_fwd(x, w, b)
    xr = x.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    br = b.float().requires_grad_(True)
    yr = F.layer_norm(xr, (H,), wr, br, 1e-5)
    assert _rel(y, yr) < 1e-2
    dy = torch.randn(rows, H, device=cuda).to(torch.bfloat16)
    dres = torch.randn(rows, H, device=cuda).to(torch.bfloat16)
    yr.backward(dy.float())
    dg = torch.full((H,), 0.5, device=cuda)
    db = torch.full((H,), -0.25, device=cuda)
    scratch = torch.empty(k.layernorm_scratch_floats(rows, H), device=cuda)
    dx = k.layernorm_bwd(x, w, mean, rstd, dy, dg, db, scratch, dres=dres)
    assert _rel(dx, xr.grad + dres.float()) < 1e-2
    assert _rel(dg - 0.5, wr.grad) < 1e-3
    assert _rel(db + 0.25, br.grad) < 1e-3
    # determinism: the same call twice gives identical bits
    dg2 = torch.full((H,), 0.5, device=cuda)
    db2 = torch.full((H,), -0.25, device=cuda)
    dx2 = k.layernorm_bwd(x, w, mean, rstd, dy, dg2, db2, scratch, dres=dres)
    assert torch.equal(dx, dx2) and torch.equal(dg, dg2) and torch.equal(db, db2)


def _sdpa_reference(qkv, mb, seq, Hl):
    import torch
    import torch.nn.functional as F
    q, k, v = qkv.float().reshape(mb, seq, 3, Hl, 128).permute(2, 0, 3, 1, 4).unbind(0)
    return q, k, v


@pytest.mark.parametrize("mb,seq,Hl", [(1, 256, 2), (2, 192, 1), (1, 1024, 4), (1, 200, 1)])
def test_attention_fwd_bwd(cuda, mb, seq, Hl):
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(1)
    qkv = torch.randn(mb * seq, 3 * Hl * 128, device=cuda).to(torch.bfloat16)
    out, lse = k.attention_fwd(qkv, mb, seq, Hl)
    qkv_r = qkv.float().requires_grad_(True)
    q, kk, v = qkv_r.reshape(mb, seq, 3, Hl, 128).permute(2, 0, 3, 1, 4).unbind(0)
    o_r = F.scaled_dot_product_attention(q, kk, v, is_causal=True)
    o_r = o_r.transpose(1, 2).reshape(mb * seq, Hl * 128)
    assert _rel(out, o_r) < 1e-2
    dout = torch.randn_like(out)
    o_r.backward(dout.float())
    dqkv = k.attention_bwd(qkv, out, dout, lse, mb, seq, Hl)
    ref = qkv_r.grad.reshape(mb * seq, 3, Hl * 128)
    got = dqkv.reshape(mb * seq, 3, Hl * 128)
    for part in range(3):
        assert _rel(got[:, part], ref[:, part]) < 2e-2, part
    dqkv2 = k.attention_bwd(qkv, out, dout, lse, mb, seq, Hl)
    assert torch.equal(dqkv, dqkv2)


@pytest.mark.parametrize("mb,seq,Hl", [(1, 128, 1), (1, 256, 2), (2, 384, 3), (1, 2048, 2)])
@pytest.mark.parametrize("impl", ["tc", "mma"])
def test_attention_fwd_impls_against_fp32(cuda, mb, seq, Hl, impl):
    """Both forward kernels (tcgen05 and mma.sync) against fp32 math, lse included."""
    import torch
    from tempname_dcu_b200.ops import kernels as k
    from tempname_dcu_b200.ops import native
    torch.manual_seed(11)
    qkv = (torch.randn(mb * seq, 3 * Hl * 128, device=cuda) * 1.5).to(torch.bfloat16)
    out, lse = k.attention_fwd(qkv, mb, seq, Hl, impl=impl)
    q, kk, v = qkv.float().reshape(mb, seq, 3, Hl, 128).permute(2, 0, 3, 1, 4).unbind(0)
    s = (q @ kk.transpose(-1, -2)) / math.sqrt(128)
    s = s.masked_fill(torch.ones(seq, seq, device=cuda, dtype=torch.bool).triu(1), float("-inf"))
    ref = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(mb * seq, Hl * 128)
    lse_ref = torch.logsumexp(s, -1) * (1.0 / math.log(2.0))
    assert _rel(out, ref) < 1e-2
    assert (lse - lse_ref).abs().max().item() < 2e-2
    assert native.read_status()[0] == 0


@pytest.mark.parametrize("mb,seq,Hl", [(1, 128, 1), (1, 256, 2), (2, 384, 3), (1, 2048, 2)])
@pytest.mark.parametrize("impl", ["tc", "mma"])
def test_attention_bwd_impls_against_fp32(cuda, mb, seq, Hl, impl):
    """Both backward paths against fp32 autograd; deterministic bits on repeat."""
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import kernels as k
    from tempname_dcu_b200.ops import native
    torch.manual_seed(12)
    qkv = torch.randn(mb * seq, 3 * Hl * 128, device=cuda).to(torch.bfloat16)
    out, lse = k.attention_fwd(qkv, mb, seq, Hl, impl="mma")
    qkv_r = qkv.float().requires_grad_(True)
    q, kk, v = qkv_r.reshape(mb, seq, 3, Hl, 128).permute(2, 0, 3, 1, 4).unbind(0)
    o_r = F.scaled_dot_product_attention(q, kk, v, is_causal=True).transpose(1, 2).reshape(mb * seq, Hl * 128)
    dout = torch.randn_like(out)
    o_r.backward(dout.float())
    dqkv = k.attention_bwd(qkv, out, dout, lse, mb, seq, Hl, impl=impl)
    ref = qkv_r.grad.reshape(mb * seq, 3, Hl * 128)
    got = dqkv.reshape(mb * seq, 3, Hl * 128)
    for part in range(3):
        assert _rel(got[:, part], ref[:, part]) < 2e-2, part
    assert torch.equal(dqkv, k.attention_bwd(qkv, out, dout, lse, mb, seq, Hl, impl=impl))
    assert native.read_status()[0] == 0


@pytest.mark.parametrize("world", [1, 2])
def test_vocab_parallel_cross_entropy(cuda, world):
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(2)
    rows, vocab, padded = 64, 1000, 1024
    full = torch.randn(rows, padded, device=cuda).to(torch.bfloat16) * 3
    targets = torch.randint(0, vocab, (rows,), device=cuda)
    local = padded // world
    stats = []
    for r in range(world):
        shard = full[:, r * local:(r + 1) * local].contiguous()
        valid = max(0, min(local, vocab - r * local))
        stats.append(k.xent_stats(shard, targets, r * local, valid))
    all_stats = torch.stack(stats)
    gstats = torch.empty(rows, 2, device=cuda)
    row_loss = torch.empty(rows, device=cuda)
    loss = torch.zeros((), device=cuda)
    k.xent_combine(all_stats, world, rows, gstats, row_loss, loss, 1.0 / rows)
    logits_r = full[:, :vocab].float().requires_grad_(True)
    ref = F.cross_entropy(logits_r, targets)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-4 * max(1, abs(ref.item()))
    grads = []
    for r in range(world):
        shard = full[:, r * local:(r + 1) * local].contiguous()
        valid = max(0, min(local, vocab - r * local))
        k.xent_grad(shard, targets, r * local, valid, gstats, 1.0 / rows)
        grads.append(shard)
    g = torch.cat(grads, 1)
    assert _rel(g[:, :vocab], logits_r.grad) < 1e-2
    assert g[:, vocab:].abs().max().item() == 0


@pytest.mark.parametrize("device_step", [False, True])
@pytest.mark.parametrize("n,split", [(10_000, 6000), (10_001, 6001)])  # vectorised / scalar kernel
def test_adamw_matches_torch(cuda, n, split, device_step):
    import torch
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(3)
    master = torch.randn(n, device=cuda)
    pa = torch.nn.Parameter(master[:split].clone())
    pb = torch.nn.Parameter(master[split:].clone())
    opt = torch.optim.AdamW([dict(params=[pa], weight_decay=0.01), dict(params=[pb], weight_decay=0.0)],
                            lr=1e-3, betas=(0.9, 0.95), eps=1e-8, foreach=False)
    m = torch.zeros(n, device=cuda)
    v = torch.zeros(n, device=cuda)
    bf = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    coef = torch.tensor([0.5], device=cuda)
    step_dev = torch.zeros((), dtype=torch.int32, device=cuda)
    total = torch.ones((), dtype=torch.float64, device=cuda)
    scratch = [torch.empty((), dtype=torch.float64, device=cuda), torch.empty((), dtype=torch.float32, device=cuda)]
    for step in range(1, 4):
        g = torch.randn(n, device=cuda)
        grad = g.clone()
        if device_step:  # the clip kernel advances the device step counter the AdamW kernel reads
            k.clip_coef(total, 1.0, scratch[0], scratch[1], step_counter=step_dev)
            k.adamw(master, grad, m, v, bf, wd_ranges=[(0, split)], lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8,
                    weight_decay=0.01, step_dev=step_dev, coef=coef)
            assert int(step_dev.item()) == step
        else:
            k.adamw(master, grad, m, v, bf, wd_ranges=[(0, split)], lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8,
                    weight_decay=0.01, step=step, coef=coef)
        assert grad.abs().max().item() == 0  # gradient reset is fused
        pa.grad, pb.grad = g[:split] * 0.5, g[split:] * 0.5
        opt.step()
    ref = torch.cat([pa.detach(), pb.detach()])
    assert _rel(master, ref) < 1e-6
    assert torch.equal(bf, master.to(torch.bfloat16))


@pytest.mark.parametrize("rows,cols,offset", [(2048, 4096, 0), (300, 12288, 0), (100, 1000, 0), (64, 514, 2)])
def test_colsum_deterministic(cuda, rows, cols, offset):
    """Column sums (bias gradients) on the 16-byte path and the 4-byte path."""
    import torch
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(8)
    base = torch.randn(rows, cols + offset, device=cuda).to(torch.bfloat16)
    x = base[:, offset:]                       # offset 2: rows 4-byte but not 16-byte aligned
    out = torch.full((cols,), 0.25, device=cuda)
    scratch = torch.empty(k.colsum_scratch_floats(rows, cols), device=cuda)
    k.colsum(x, out, scratch, accumulate=True)
    ref = x.double().sum(0) + 0.25
    assert (out.double() - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())
    out2 = torch.full((cols,), 0.25, device=cuda)
    k.colsum(x, out2, scratch, accumulate=True)
    assert torch.equal(out, out2)


def test_sumsq_and_clip(cuda):
    import torch
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(4)
    g = torch.randn(123_457, device=cuda)
    partial = torch.empty(k.sumsq_partials_count(), dtype=torch.float64, device=cuda)
    total = torch.empty((), dtype=torch.float64, device=cuda)
    k.sumsq(g, partial, total)
    ref = g.double().square().sum()
    assert abs(total.item() - ref.item()) < 1e-9 * ref.item()
    norm = torch.empty((), dtype=torch.float64, device=cuda)
    coef = torch.empty((), dtype=torch.float32, device=cuda)
    finite = torch.ones((), dtype=torch.int32, device=cuda)
    k.clip_coef(total, 1.0, norm, coef, None, finite)
    assert abs(norm.item() - math.sqrt(ref.item())) < 1e-6 * math.sqrt(ref.item())
    assert abs(coef.item() - 1.0 / (math.sqrt(ref.item()) + 1e-6)) < 1e-6
    assert finite.item() == 1


def test_embedding_fwd_bwd(cuda):
    import torch
    import torch.nn.functional as F
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(5)
    vocab, H, seq, rows = 64, 256, 16, 32
    table = torch.randn(vocab, H, device=cuda).to(torch.bfloat16)
    pos = torch.randn(seq, H, device=cuda).to(torch.bfloat16)
    tokens = torch.randint(0, vocab, (rows,), device=cuda)
    out = torch.empty(rows, H, dtype=torch.bfloat16, device=cuda)
    # shard 1 of 2: vocab rows [32, 64)
    k.embedding_fwd(tokens, table[32:].contiguous(), 32, out, pos, 0, seq)
    mask = ((tokens >= 32) & (tokens < 64)).unsqueeze(1)
    ref = F.embedding((tokens - 32).clamp(0, 31), table[32:].float()) * mask + pos.float()[torch.arange(rows, device=cuda) % seq]
    assert _rel(out, ref) < 1e-2
    dy = torch.randn(rows, H, device=cuda).to(torch.bfloat16)
    st, order = torch.sort(tokens, stable=True)
    grad = torch.zeros(32, H, device=cuda)
    k.embedding_bwd(st, order, dy, 32, 32, grad)
    ref_g = torch.zeros(vocab, H, device=cuda)
    ref_g.index_add_(0, tokens, dy.float())
    assert _rel(grad, ref_g[32:]) < 1e-5
    gp = torch.zeros(seq, H, device=cuda)
    k.position_bwd(dy, 0, seq, gp)
    ref_p = torch.zeros(seq, H, device=cuda)
    ref_p.index_add_(0, torch.arange(rows, device=cuda) % seq, dy.float())
    assert _rel(gp, ref_p) < 1e-5


@pytest.mark.parametrize("n,vocab", [(1, 10), (37, 5), (2048, 50257), (3000, 100), (16384, 50304)])
def test_sort_tokens_is_a_stable_sort(cuda, n, vocab):
    import torch
    from tempname_dcu_b200.ops import kernels as k
    torch.manual_seed(n)
    tokens = torch.randint(0, vocab, (n,), device=cuda)
    st, order = k.sort_tokens(tokens)
    ref_t, ref_o = torch.sort(tokens, stable=True)
    assert torch.equal(st, ref_t) and torch.equal(order, ref_o)


def test_native_library_is_the_in_tree_build(cuda):
    from pathlib import Path
    from tempname_dcu_b200.ops import _build, native
    native.lib()
    loaded = Path(native.LOADED_PATH).resolve()
    assert loaded == _build.paths(_build.debug_requested())[0].resolve()
    assert loaded.parent == (Path(__file__).resolve().parents[1] / "tempname_dcu_b200" / "_native")
