"""The CPU oracle against the golden vectors the reference itself produced (tests/golden/make_golden.py):
store_kvcache under the Triton interpreter and verify_drafts on CPU.  Plus self-checks of the FP32 attention
restatement on cases small enough to spell out by hand."""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden


def _tensor(raw, dtype):
    if dtype == "torch.bfloat16":
        return torch.from_numpy(raw.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(raw.copy())


def _scatter_inputs(c):
    N, KVH, D, NB = c["shape"].tolist()
    dt = str(c["dtype"])
    kb = _tensor(c["key_base"], dt).reshape(-1)
    vb = _tensor(c["value_base"], dt).reshape(-1)
    key = kb.as_strided((N, KVH, D), (int(c["key_row_stride"]), D, 1), int(c["key_offset"]))
    value = vb.as_strided((N, KVH, D), (int(c["value_row_stride"]), D, 1), int(c["value_offset"]))
    kc = _tensor(c["k_in"], dt).view(NB, 256, KVH, D).clone()
    vc = _tensor(c["v_in"], dt).view(NB, 256, KVH, D).clone()
    slots = torch.from_numpy(c["slots"].astype(np.int32))
    return key, value, kc, vc, slots, dt


SCATTER = load_golden("scatter_golden.npz")
ACCEPT = load_golden("accept_golden.npz")


@pytest.mark.parametrize("case", sorted(SCATTER))
def test_scatter_c_oracle_matches_reference(case):
    c = SCATTER[case]
    key, value, kc, vc, slots, dt = _scatter_inputs(c)
    assert oracle.store_kvcache(key, value, kc, vc, slots) == 0
    assert torch.equal(kc.view(torch.uint8 if False else kc.dtype), _tensor(c["k_out"], dt).view(kc.shape))
    assert torch.equal(vc, _tensor(c["v_out"], dt).view(vc.shape))


@pytest.mark.parametrize("case", sorted(SCATTER))
def test_scatter_torch_oracle_matches_reference(case):
    c = SCATTER[case]
    key, value, kc, vc, slots, dt = _scatter_inputs(c)
    oracle.store_kvcache_ref(key, value, kc, vc, slots)
    assert torch.equal(kc, _tensor(c["k_out"], dt).view(kc.shape))
    assert torch.equal(vc, _tensor(c["v_out"], dt).view(vc.shape))


def test_scatter_oracle_counts_out_of_range():
    key = torch.randn(3, 2, 8)
    kc = torch.zeros(1, 256, 2, 8)
    vc = torch.zeros_like(kc)
    assert oracle.store_kvcache(key, key, kc, vc, torch.tensor([0, 256, -5], dtype=torch.int32)) == 2


@pytest.mark.parametrize("case", sorted(ACCEPT))
def test_accept_oracles_match_reference(case):
    c = ACCEPT[case]
    a, t = oracle.greedy_accept(c["target"], c["drafts"], c["num_drafts"])
    assert np.array_equal(a, c["num_accepted"]) and np.array_equal(t, c["next_token"])
    a, t = oracle.greedy_accept_ref(c["target"], c["drafts"], c["num_drafts"])
    assert np.array_equal(a, c["num_accepted"]) and np.array_equal(t, c["next_token"])


def test_accept_hand_case_values():
    c = ACCEPT["hand"]
    assert c["num_accepted"].tolist() == [3, 1, 0, 1] and c["next_token"].tolist() == [6, 4, 3, 4]


def _naive(q, ks, vs, scale):
    """Loop-by-loop restatement for tiny cases: q [n, H, D], ks/vs [L, KVH, D]."""
    n, H, D = q.shape
    L, KVH, _ = ks.shape
    out = torch.zeros(n, H, D, dtype=torch.float64)
    for i in range(n):
        for h in range(H):
            kh = h // (H // KVH)
            vis = [j for j in range(L) if j <= L - n + i]
            if not vis:
                continue
            s = [float(q[i, h].double() @ ks[j, kh].double()) * scale for j in vis]
            m = max(s)
            w = [math.exp(x - m) for x in s]
            tot = sum(w)
            out[i, h] = sum(wj * vs[j, kh].double() for wj, j in zip(w, vis)) / tot
    return out


@pytest.mark.parametrize("n,L", [(1, 5), (3, 7), (4, 4), (2, 1), (3, 0)])
def test_attention_oracle_matches_naive_loops(n, L):
    g = torch.Generator().manual_seed(n * 31 + L)
    H, KVH, D = 4, 2, 8
    q = torch.randn(n, H, D, generator=g)
    k = torch.randn(max(L, 1), KVH, D, generator=g)[:L]
    v = torch.randn(max(L, 1), KVH, D, generator=g)[:L]
    cu_q = torch.tensor([0, n], dtype=torch.int32)
    cu_k = torch.tensor([0, L], dtype=torch.int32)
    got = oracle.varlen_attention_ref(q, k, v, cu_q, cu_k, 0.3)
    ref = _naive(q, k, v, 0.3)
    assert torch.allclose(got.double(), ref, atol=1e-5)


def test_paged_oracle_equals_contiguous_oracle():
    """The paged gather (block table, slot rule of model_runner.py:338) sees the same keys as contiguous rows."""
    from nvattn.workloads import config1
    b = config1(0)["batch"]
    q = b.q.view(4, 1, 16, 128)
    paged = oracle.paged_attention_ref(q, b.k_cache, b.v_cache, b.context_lens, b.block_tables, b.scale)
    for i, L in enumerate(b.meta["lens"]):
        nblk = (L + 255) // 256
        ks = b.k_cache[b.block_tables[i, :nblk].long()].reshape(-1, 8, 128)[:L]
        vs = b.v_cache[b.block_tables[i, :nblk].long()].reshape(-1, 8, 128)[:L]
        cu = torch.tensor([0, 1], dtype=torch.int32)
        ref = oracle.varlen_attention_ref(q[i], ks, vs, cu, torch.tensor([0, L], dtype=torch.int32), b.scale)
        assert torch.allclose(paged[i], ref, atol=1e-6)


def test_config1_slots_follow_block_rule():
    from nvattn.workloads import config1
    b = config1(0)["batch"]
    for i, L in enumerate([37, 256, 513, 1000]):
        p = L - 1
        assert int(b.slot_mapping[i]) == int(b.block_tables[i, p // 256]) * 256 + p % 256
    used = [int(x) for row in b.block_tables for x in row if x >= 0]
    assert len(used) == len(set(used)) and all(0 <= x < 64 for x in used)


# ------------------------------------------------------------------ attention pinned to flash-attn 2.8.3
FA2 = None


def _fa2():
    global FA2
    if FA2 is None:
        import numpy as np
        import os
        from conftest import REPO
        z = np.load(os.path.join(REPO, "tests", "golden", "attention_fa2_golden.npz"))
        FA2 = {k: z[k] for k in z.files}
    return FA2


def fa2_case(name):
    """(inputs rebuilt from the generator's seed, flash-attn's bf16 output) for one golden case."""
    import sys
    import os
    from conftest import REPO
    sys.path.insert(0, os.path.join(REPO, "tests", "golden"))
    import make_golden_fa2 as mg
    kind, args = next((k, a) for n, k, a in mg.CASES if n == name)
    b = mg.build(kind, args)
    g = _fa2()
    assert np.allclose(mg.checksum(b), g[f"{name}/checksum"], rtol=1e-9, atol=1e-6), "regenerated inputs drifted"
    out = torch.from_numpy(g[f"{name}/out"].view(np.int16).copy()).view(torch.bfloat16)
    return kind, args, b, out


FA2_CASES = ["decode", "verify_k3", "verify_k8_padded", "mixed_paged", "prefill_contiguous"]


@pytest.mark.parametrize("name", FA2_CASES)
def test_attention_oracle_matches_flash_attn(name):
    """The FP32 restatement against the reference's own attention library (flash-attn 2.8.3 on B200, called as
    attention.py calls it), within the bf16 tolerance: pins the attention oracle."""
    from conftest import assert_attn_close
    kind, args, b, out = fa2_case(name)
    if kind == "paged_decode":
        B, n = b.num_seqs, b.q_per_seq
        ref = oracle.paged_attention_ref(b.q.view(B, n, 8, 128), b.k_cache, b.v_cache, b.context_lens,
                                         b.block_tables, b.scale).reshape(B * n, 8, 128)
    elif b.meta["paged"]:
        ref = oracle.varlen_attention_ref(b.q, None, None, b.cu_seqlens_q, b.cu_seqlens_k, b.scale,
                                          block_tables=b.block_tables, k_cache=b.k_cache, v_cache=b.v_cache)
    else:
        ref = oracle.varlen_attention_ref(b.q, b.k_new, b.v_new, b.cu_seqlens_q, b.cu_seqlens_k, b.scale)
    assert_attn_close(out, ref, f"flash-attn vs oracle: {name}")
