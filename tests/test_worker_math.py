"""Worker helpers on CPU (reference: tests/test_worker_math.py): the
closed-block selective reference, role plans reaching the right operators,
the torch independent codec against the FP64 oracle, tensor-hash bit
sensitivity, and the torch restatement of the FP8 quantizer used as the
fp8-mma reference."""
import torch

from tempname_dcu_b200 import reference
from tempname_dcu_b200.mapping import ARMS
from tempname_dcu_b200.worker import independent_codec, reduce_reference_sources, tensor_sha


def test_closed_block_selective_reference():
    torch.manual_seed(0)
    world, per, chunk, n = 2, 3, 128, 256
    sources = torch.randn(world, per * chunk, n).to(torch.bfloat16)
    mask = [True, False, True, False, False, True]  # physical blocks; rank 1 owns 3..5
    plain, coded = reduce_reference_sources(sources, 1, True, mask, chunk)
    for w in range(per):
        blk = slice(w * chunk, (w + 1) * chunk)
        if mask[per + w]:
            assert not torch.equal(coded[blk], plain[blk])
        else:
            assert torch.equal(coded[blk], plain[blk])
    # the local source (rank 1) is never coded: with one source the sums agree exactly
    one = sources[:1]
    p1, c1 = reduce_reference_sources(one, 0, True, [True] * per, chunk)
    assert torch.equal(p1, c1)


def test_role_plans_reach_the_right_operators():
    from tempname_dcu_b200.models.config import SMALL_CONFIG
    from tempname_dcu_b200.models.gpt import GPT
    seen = []

    def factory(m, n, k, group, arm, chunk_rows, plan):
        seen.append((k, arm, plan))
        return object()
    roles = dict(attn=dict(tag="attn-plan"), mlp=dict(tag="mlp-plan"))
    cfg = dict(SMALL_CONFIG)
    GPT(cfg, ARMS[4], device="cpu", operator_factory=factory, execution_plan=dict(roles=roles), materialize=False)
    assert len(seen) == 2 * cfg["layers"]
    for i, (k, arm, plan) in enumerate(seen):
        role = "attn" if i % 2 == 0 else "mlp"
        assert k == (cfg["hidden"] if role == "attn" else cfg["ffn"]) and arm == ARMS[4]
        assert plan == roles[role]
    seen.clear()
    GPT(cfg, ARMS[1], device="cpu", operator_factory=factory, execution_plan=dict(roles=roles), materialize=False)
    assert all(plan is None for _, _, plan in seen)


def test_torch_codec_matches_the_fp64_oracle():
    torch.manual_seed(3)
    x = (torch.randn(8 * 128) * torch.logspace(-2, 2, 8 * 128)).to(torch.bfloat16)
    ours = independent_codec(x).float()
    oracle = torch.tensor(reference.decode(reference.encode([float(v) for v in x.float()])))
    assert float((ours - oracle).norm() / oracle.norm()) <= 0.02


def test_tensor_hash_is_bit_sensitive():
    x = torch.randn(64, 64).to(torch.bfloat16)
    y = x.clone()
    assert tensor_sha(x) == tensor_sha(y)
    y.view(torch.int16)[3, 5] ^= 1  # one mantissa bit
    assert tensor_sha(x) != tensor_sha(y)


def test_fp8_reference_dequantizes_close_to_the_input():
    from tempname_dcu_b200.ops import mx
    torch.manual_seed(4)
    x = torch.randn(128, 256).to(torch.bfloat16)
    values, e = mx.quantize_reference(x)
    deq = (values.view(128, -1, 32) * torch.exp2(e.float()).unsqueeze(-1)).view(128, 256)
    assert float((deq - x.float()).norm() / x.float().norm()) < 0.04


def test_trace_categories_bucket_kernel_names():
    from tempname_dcu_b200.utils.trace import categorize
    kernels = [dict(name="void tdb::rs::gemm_rs_kernel<256, true>(...)", us=10.0, count=2),
               dict(name="tdb::rs::rs_reduce_kernel(tdb::rs::Params, int*)", us=5.0, count=2),
               dict(name="void tdb::aggemm::ag_gemm2_kernel<true, 11, false>(...)", us=7.0, count=1),
               dict(name="void tdb::gemm::gemm2_kernel<true, true, 6>(...)", us=3.0, count=1),
               dict(name="ncclDevKernel_ReduceScatter_Sum_bf16_RING_LL(...)", us=1.0, count=1),
               dict(name="tdb::aggemm::push_advance_kernel(unsigned int*)", us=0.25, count=1),
               dict(name="tdb::embx::push_fwd_kernel(tdb::embx::Params, ...)", us=2.0, count=1),
               dict(name="something_else", us=0.5, count=1)]
    cats = categorize(kernels)
    assert cats["fused GEMM -> reduce-scatter"] == (15.0, 4)
    assert cats["fused all-gather -> GEMM"] == (7.25, 2)
    assert cats["embedding"] == (2.0, 1)
    assert cats["GEMM (tcgen05)"] == (3.0, 1) and cats["NCCL"] == (1.0, 1) and cats["other"] == (0.5, 1)


def test_fused_path_rooflines_for_gpt67b_tp8():
    from tempname_dcu_b200.models.config import BENCH_CONFIG
    from tempname_dcu_b200.ops import roofline as rf
    paths = {p["name"]: p for p in rf.fused_paths(BENCH_CONFIG, 8)}
    assert abs(paths["qkv.fwd"]["flops"] - 25.77e9) < 0.01e9 and paths["qkv.fwd"]["link_bytes"] == 14_680_064
    assert abs(paths["fc2.fwd"]["flops"] - 34.36e9) < 0.01e9
    taco = {p["name"]: p for p in rf.fused_paths(BENCH_CONFIG, 8, taco=True)}
    assert taco["attn_out.fwd"]["link_bytes"] == 7_798_784  # the reference's TACO byte budget
    us, bound = rf.roofline_us(paths["attn_out.fwd"], 1651.0, 770.0)
    assert bound == "link" and abs(us - 14_680_064 / 770e3) < 1e-9
    # per step: 8 micro-batches x (32 layers x 8 paths + LM head fwd / dgrad)
    total = rf.step_roofline(BENCH_CONFIG, 8, tflops=1651.0, nvlink_gbs=770.0)
    per_layer = sum(rf.roofline_us(p, 1651.0, 770.0)[0] for p in rf.fused_paths(BENCH_CONFIG, 8))
    head = sum(rf.roofline_us(p, 1651.0, 770.0)[0] for p in rf.head_paths(BENCH_CONFIG, 8))
    assert abs(total - 8 * (32 * per_layer + head)) < 1e-6
