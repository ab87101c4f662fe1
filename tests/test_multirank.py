"""The multi-GPU path on CPU: world-size-2 gloo ranks.  nano-vllm splits attention by heads across tensor-parallel
ranks (qwen3.py:29-39, model_runner.py:251); each rank attends over its own kv-head shard of the paged cache and
needs no collective.  Here each rank computes its shard with the oracle and the shards are gathered and compared
with the unsharded computation; the max-over-ranks reduction bench.py uses for timings is checked too."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, q):
    try:
        import sys
        here = os.path.dirname(os.path.abspath(__file__))
        sys.path.insert(0, os.path.dirname(here))
        sys.path.insert(0, os.path.join(os.path.dirname(here), "nano-vllm-spec-decode_b200"))
        import oracle
        from nvattn.workloads import paged_decode_batch, varlen_batch, shard_heads
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        # decode / verify shard
        full = paged_decode_batch([300, 70, 513], 3, 32, 8, 128, 16, 0.5, seed=5, dtype=torch.float32)
        sh = shard_heads(full, rank, world)
        o = oracle.paged_attention_ref(sh.q.view(3, 3, -1, 128), sh.k_cache, sh.v_cache, sh.context_lens,
                                       sh.block_tables, sh.scale)
        parts = [torch.empty_like(o) for _ in range(world)]
        dist.all_gather(parts, o)
        ref = oracle.paged_attention_ref(full.q.view(3, 3, 32, 128), full.k_cache, full.v_cache, full.context_lens,
                                         full.block_tables, full.scale)
        ok_decode = torch.allclose(torch.cat(parts, dim=2), ref, atol=1e-5)
        # varlen shard (prefill chunk over a paged prefix + decode rows)
        fv = varlen_batch([1, 40, 2], [100, 300, 50], 32, 8, 128, 16, 0.5, seed=6, dtype=torch.float32)
        sv = shard_heads(fv, rank, world)
        ov = oracle.varlen_attention_ref(sv.q, None, None, sv.cu_seqlens_q, sv.cu_seqlens_k, sv.scale,
                                         block_tables=sv.block_tables, k_cache=sv.k_cache, v_cache=sv.v_cache)
        pv = [torch.empty_like(ov) for _ in range(world)]
        dist.all_gather(pv, ov)
        rv = oracle.varlen_attention_ref(fv.q, None, None, fv.cu_seqlens_q, fv.cu_seqlens_k, fv.scale,
                                         block_tables=fv.block_tables, k_cache=fv.k_cache, v_cache=fv.v_cache)
        ok_varlen = torch.allclose(torch.cat(pv, dim=1), rv, atol=1e-5)
        # bench.py's timing rule: the slowest rank's time is the step time
        t = torch.tensor([1.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ok_max = float(t) == float(world)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok_decode, ok_varlen, ok_max))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), False, False))


@pytest.mark.parametrize("world", [2])
def test_head_shards_need_no_collective(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok_decode, ok_varlen, ok_max in results:
        assert ok_decode is True, (rank, ok_decode)
        assert ok_varlen and ok_max, rank
