"""Sparse embedding exchange (csrc/embed_exchange.cu) on 2 GPUs against the
dense NCCL path it replaces, bit for bit:

* forward: masked lookup + NCCL reduce-scatter + positions == exchange;
* backward: the table gradient from the rows the exchange delivers ==
  the one from the NCCL all-gathered rows;
* several calls in a row (both slot parities) and replays of a captured CUDA
  graph with changing tokens.

Child processes over NCCL (NVLS off); skipped with fewer than two GPUs.
"""
import os

import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, init_file, result_path):
    import json
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    from tempname_dcu_b200.ops import kernels as K
    from tempname_dcu_b200.ops import native
    from tempname_dcu_b200.parallel.embedding_exchange import EmbeddingExchange
    from tempname_dcu_b200.parallel.tp import TPGroup
    out = {"fwd": [], "bwd": [], "graph": []}
    try:
        tp = TPGroup(dist.group.WORLD)
        vocab, H, ml, seq = 1024, 512, 256, 512
        local = vocab // world
        start = rank * local
        gen = torch.Generator(device="cuda").manual_seed(5)
        table = torch.randn(local, H, device="cuda", generator=torch.Generator(device="cuda").manual_seed(rank)).to(torch.bfloat16)
        pos = torch.randn(seq, H, device="cuda", generator=gen).to(torch.bfloat16)
        ex = EmbeddingExchange(tp, ml, H, local)

        def dense(tokens):
            full = torch.empty(world * ml, H, dtype=torch.bfloat16, device="cuda")
            K.embedding_fwd(tokens, table, start, full)
            x = tp.scatter_sum(full)
            K.add_positions(x, pos, rank * ml, seq)
            return x

        def grads(tokens, dfull):
            g = torch.zeros(local, H, device="cuda")
            st, order = K.sort_tokens(tokens)
            K.embedding_bwd(st, order, dfull, start, local, g)
            return g

        for call in range(4):
            tokens = torch.randint(0, vocab, (world * ml,), device="cuda", generator=gen)
            x = ex.forward(tokens, table, start, pos, rank * ml, seq)
            out["fwd"].append(bool(torch.equal(x, dense(tokens))))
            dy = torch.randn(ml, H, device="cuda", generator=torch.Generator(device="cuda").manual_seed(10 + rank + 7 * call)).to(torch.bfloat16)
            dfull = torch.full((world * ml, H), float("nan"), dtype=torch.bfloat16, device="cuda")
            ex.backward(tokens, dy, start, dfull)
            out["bwd"].append(bool(torch.equal(grads(tokens, dfull), grads(tokens, tp.gather(dy)))))
        # captured: three exchange calls per replay (odd, so the slot parity changes between replays)
        tok = torch.zeros(world * ml, dtype=torch.int64, device="cuda")
        xs = [torch.empty(ml, H, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for x in xs:
                ex.forward(tok, table, start, pos, rank * ml, seq, out=x)
        for rep in range(3):
            tok.copy_(torch.randint(0, vocab, (world * ml,), device="cuda", generator=gen))
            graph.replay()
            torch.cuda.synchronize()
            ref = dense(tok)
            out["graph"].append(all(bool(torch.equal(x, ref)) for x in xs))
        del graph
        torch.cuda.synchronize()
        native.raise_on_status()
        ex.close()
    finally:
        if rank == 0:
            with open(result_path, "w") as fh:
                json.dump(out, fh)
        dist.destroy_process_group()


def test_embedding_exchange_matches_dense_nccl_path(tmp_path):
    import json
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    path = str(tmp_path / "result.json")
    # TDB_TEST_WORLD runs the same checks on more ranks (up to the visible GPUs)
    world = min(int(os.environ.get("TDB_TEST_WORLD", "2")), torch.cuda.device_count())
    mp.spawn(_worker, args=(world, str(tmp_path / "rendezvous"), path), nprocs=world, join=True)
    res = json.load(open(path))
    assert res["fwd"] and all(res["fwd"]), res
    assert res["bwd"] and all(res["bwd"]), res
    assert res["graph"] and all(res["graph"]), res
