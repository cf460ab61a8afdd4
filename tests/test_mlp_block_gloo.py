"""One GPT-6.7B-shaped tensor-parallel MLP block on two CPU gloo ranks (no GPU):
hidden 4096, FFN 16384, seq 2048, batch 1, fp32, weights N(0, 0.02), inputs
N(0, 1).  Sequence-parallel all-gather -> FC1 + exact GELU -> FC2 ->
reduce-scatter, where each rank's FC2 partial is cut into 128-row blocks and
delivered in the production order of the common tile mapping
(``mapping.schedule``, interleaved arm), then summed in source order.  Checked
against the unsplit block; then the TACO round trip of a remote contribution
(the torch independent codec against the FP64 oracle) and the selective arm's
closed-block error on the real partials.

Reference parity: the reference's 2-rank gloo model test
(tests/test_model_contract.py:159-165) and its worker math tests
(tests/test_worker_math.py:13-65).
"""
import json
import os

H, F, SEQ, W, CHUNK = 4096, 16384, 2048, 2, 128


def _worker(rank, world, init_file, result_path):
    import torch
    import torch.distributed as dist
    import torch.nn.functional as Fn
    from tempname_dcu_b200 import reference
    from tempname_dcu_b200.mapping import ARMS, schedule
    from tempname_dcu_b200.planning import make_role
    from tempname_dcu_b200.worker import independent_codec, reduce_reference_sources
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // world))
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    out = {}
    try:
        gen = torch.Generator().manual_seed(1234)  # identical full tensors on every rank
        x = torch.randn(SEQ, H, generator=gen)
        w1 = torch.randn(F, H, generator=gen) * 0.02
        w2 = torch.randn(H, F, generator=gen) * 0.02
        rows, cols = SEQ // world, F // world
        # sequence-parallel input -> all-gather
        parts = [torch.empty(rows, H) for _ in range(world)]
        dist.all_gather(parts, x[rank * rows:(rank + 1) * rows].contiguous())
        x_full = torch.cat(parts)
        # column-parallel FC1 + GELU, row-parallel FC2 (local partial of every output row)
        h = Fn.gelu(x_full @ w1[rank * cols:(rank + 1) * cols].t())
        partial = h @ w2[:, rank * cols:(rank + 1) * cols].t()
        # deliver 128-row blocks in the common mapping's production order
        order = schedule(SEQ, H, cols, world, CHUNK, ARMS[2])
        received = torch.zeros(world, rows, H)  # [source, local row, col]
        for item in order:
            block = partial[item["row"]:item["row"] + CHUNK].contiguous()
            blocks = [torch.empty_like(block) for _ in range(world)]
            dist.all_gather(blocks, block)  # every rank produces the same physical block id in this slot
            if item["destination"] == rank:
                for s in range(world):
                    received[s, item["within"] * CHUNK:(item["within"] + 1) * CHUNK] = blocks[s]
        mine = received.sum(0)
        ref = Fn.gelu(x_full @ w1.t()) @ w2.t()
        ref_rows = ref[rank * rows:(rank + 1) * rows]
        out["mlp_rel"] = float((mine - ref_rows).norm() / ref_rows.norm())
        out["destinations"] = sorted({(it["destination"], it["within"], it["physical"]) for it in order})
        # TACO round trip of a remote contribution: torch codec vs the FP64 oracle
        remote = received[(rank + 1) % world, :CHUNK].to(torch.bfloat16)
        sample = remote.reshape(-1)[:4 * 128]
        torch_rt = independent_codec(sample).float()
        oracle_rt = torch.tensor(reference.decode(reference.encode([float(v) for v in sample.float()])))
        out["codec_vs_oracle"] = float((torch_rt - oracle_rt).norm() / oracle_rt.norm())
        out["codec_vs_input"] = float((torch_rt - sample.float()).norm() / sample.float().norm())
        # selective arm: the masked receiver blocks carry TACO on their remote sources
        per = rows // CHUNK
        mask = [(i % 3) == 0 for i in range(world * per)]
        make_role(SEQ, H, cols, world, CHUNK, mask=mask)  # a legal plan for this shape
        plain, coded = reduce_reference_sources(received.to(torch.bfloat16), rank, True, mask, CHUNK)
        errs, same = [], []
        for w in range(per):
            blk = slice(w * CHUNK, (w + 1) * CHUNK)
            if mask[rank * per + w]:
                errs.append(float((coded[blk].float() - plain[blk].float()).norm() / plain[blk].float().norm()))
            else:
                same.append(bool(torch.equal(coded[blk], plain[blk])))
        out["selective_block_err"] = errs
        out["unselected_bitwise"] = same
        out["selective_total_err"] = float((coded.float() - ref_rows).norm() / ref_rows.norm())
    finally:
        with open(f"{result_path}.{rank}", "w") as fh:
            json.dump(out, fh)
        dist.destroy_process_group()


def test_tp_mlp_block_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    path = str(tmp_path / "result")
    mp.spawn(_worker, args=(W, str(tmp_path / "rendezvous"), path), nprocs=W, join=True)
    for rank in range(W):
        res = json.load(open(f"{path}.{rank}"))
        assert res["mlp_rel"] < 1e-5, res["mlp_rel"]
        # the common mapping sends physical block p to destination p // per, slot p % per
        per = SEQ // W // CHUNK
        assert res["destinations"] == sorted([d, p % per, p] for p in range(W * per) for d in [p // per])
        assert res["codec_vs_oracle"] <= 0.02, res["codec_vs_oracle"]
        assert res["codec_vs_input"] < 0.05, res["codec_vs_input"]
        assert res["selective_block_err"] and all(0 < e < 0.05 for e in res["selective_block_err"])
        assert res["unselected_bitwise"] and all(res["unselected_bitwise"])
        assert res["selective_total_err"] < 0.05
