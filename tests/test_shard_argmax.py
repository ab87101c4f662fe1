"""Greedy verify over vocabulary shards on the CPU: the numpy restatement (oracle/argmax.py) pinned to torch's
argmax and to the reference's verify_drafts golden vectors, the sharded merge equal to the unsharded rule at
TP 1/2/4/8, the gather of per-rank keys between world-size-2 gloo ranks, and the host-side TP > 1 speculative
plumbing of nvattn.nanovllm_dropin (Sequence pickling, Config checks)."""
import os
import pickle
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import argmax as am
from conftest import load_golden, REPO, PKG

ACCEPT = load_golden("accept_golden.npz")


def _tricky_logits(rows, vocab, seed):
    """bf16-valued logits with many exact ties (few distinct values), -0/+0 ties and NaN rows."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-8, 8, (rows, vocab), generator=g).float() * 0.25
    x = x.to(torch.bfloat16).float()
    if rows > 3:
        x[1] = 0.0
        x[1, ::3] = -0.0            # +0 and -0 tie: the first index wins
        x[2, vocab // 2] = float("nan")
        x[2, vocab - 1] = float("nan")
        x[3] = float("-inf")
    return x


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_argmax_follows_torch(seed):
    x = _tricky_logits(16, 999, seed)
    assert np.array_equal(am.argmax_ref(x.numpy()), x.argmax(dim=-1).numpy())


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_sharded_merge_equals_unsharded(tp):
    vocab = 8 * 96
    x = _tricky_logits(24, vocab, tp).numpy()
    shard = vocab // tp
    keys = np.stack([am.shard_argmax_keys(x[:, r * shard:(r + 1) * shard], r * shard) for r in range(tp)])
    assert np.array_equal(am.merge_keys(keys), am.argmax_ref(x))


@pytest.mark.parametrize("case", sorted(ACCEPT))
@pytest.mark.parametrize("tp", [1, 2, 4])
def test_accept_from_shards_matches_reference_golden(case, tp):
    """verify_drafts' golden cases (one-hot logits at the target ids), the logits split into tp vocabulary shards."""
    c = ACCEPT[case]
    t = c["target"].astype(np.int64)
    S, K1 = t.shape
    vocab = (int(t.max()) // (4 * tp) + 1) * 4 * tp
    logits = np.zeros((S * K1, vocab), dtype=np.float32)
    logits[np.arange(S * K1), t.reshape(-1)] = 1.0
    shard = vocab // tp
    keys = np.stack([am.shard_argmax_keys(logits[:, r * shard:(r + 1) * shard], r * shard) for r in range(tp)])
    acc, nxt = am.accept_from_keys(keys.reshape(tp, S, K1), c["drafts"].reshape(S, K1 - 1), c["num_drafts"])
    assert acc.tolist() == c["num_accepted"].tolist() and nxt.tolist() == c["next_token"].tolist()


def _gather_worker(rank, world, port, q):
    try:
        sys.path.insert(0, REPO)
        from oracle import argmax as am_
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        x = _tricky_logits(40, 512, 7).numpy()
        shard = 512 // world
        keys = torch.from_numpy(am_.shard_argmax_keys(x[:, rank * shard:(rank + 1) * shard], rank * shard)
                                .view(np.int64))
        gathered = [torch.empty_like(keys) for _ in range(world)] if rank == 0 else None
        dist.gather(keys, gathered, 0)    # the exchange install_greedy_argmax makes (8 bytes per row and rank)
        if rank == 0:
            merged = am_.merge_keys(torch.stack(gathered).numpy().view(np.uint64))
            q.put(bool(np.array_equal(merged, am_.argmax_ref(x))))
        dist.destroy_process_group()
    except Exception as e:    # report instead of hanging the parent
        q.put(repr(e))


def test_gather_of_shard_keys_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert q.get(timeout=10) is True


_DROPIN_CHECK = r"""
import os, pickle, sys, tempfile
sys.path.insert(0, sys.argv[1])
from nvattn import e2e, nanovllm_dropin
e2e.ensure_reference_importable()
from nanovllm.engine.sequence import Sequence
from nanovllm.config import Config
from nanovllm.sampling_params import SamplingParams
d = e2e.write_model_dir(tempfile.mkdtemp())
try:
    Config(d, tensor_parallel_size=2, speculative_method="ngram")
    raise SystemExit("the reference accepted TP 2 with n-gram drafting")
except AssertionError:
    pass
nanovllm_dropin.install_tp_speculative()
cfg = Config(d, tensor_parallel_size=2, speculative_method="ngram", num_speculative_tokens=4)
assert cfg.tensor_parallel_size == 2
for bad in (dict(speculative_method="draft", draft_model=d), dict(speculative_method="ngram", enable_mixed_batching=True)):
    try:
        Config(d, tensor_parallel_size=2, **bad)
        raise SystemExit(f"accepted {bad}")
    except AssertionError:
        pass
seq = Sequence(list(range(300)), SamplingParams(temperature=0.0, max_tokens=8))
seq.is_prefill = False
seq.append_token(7)
seq.draft_token_ids = [11, 12, 13]
w = pickle.loads(pickle.dumps(seq))
assert w.draft_token_ids == [11, 12, 13] and w.last_token == 7 and w.temperature == 0.0, vars(w)
assert w.num_tokens == 301 and w.token_ids == []
seq.is_prefill = True
w = pickle.loads(pickle.dumps(seq))
assert w.token_ids == seq.token_ids and w.draft_token_ids == []
print("ok")
"""


def test_tp_speculative_host_plumbing():
    """install_tp_speculative on the reference's own Config and Sequence (in a fresh process: it patches them)."""
    if not os.path.isdir(os.path.join(REPO, "baseline", "_ref", "nanovllm")):
        pytest.skip("the reference is not installed under baseline/_ref")
    r = subprocess.run([sys.executable, "-c", _DROPIN_CHECK, PKG], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
