"""The fused attention prologue's CPU restatement (oracle/prologue.py) pinned to the reference's own RMSNorm and
rotary layers (golden vectors of tests/golden/make_golden_prologue.py): bit for bit, and the cos / sin table
byte-identical to the reference's."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import prologue
from conftest import load_golden

GOLD = load_golden("prologue_golden.npz")


def bf16(a):
    return torch.from_numpy(a).view(torch.bfloat16)


def case_inputs(c):
    T, H, KVH, max_pos = (int(x) for x in c["geometry"])
    table = prologue.rope_table(128, max_pos, float(c["base"][0]))
    return T, H, KVH, table, bf16(c["qkv"]), torch.from_numpy(c["positions"]), bf16(c["q_w"]), bf16(c["k_w"])


@pytest.mark.parametrize("case", sorted(GOLD))
def test_prologue_oracle_matches_reference_layers(case):
    c = GOLD[case]
    T, H, KVH, table, qkv, pos, qw, kw = case_inputs(c)
    assert hashlib.sha256(table.numpy().tobytes()).digest() == bytes(c["table_sha256"])
    q, k, v = prologue.qk_prologue_ref(qkv, pos, table, qw, kw, 1e-6, H, KVH)
    assert torch.equal(q.reshape(T, -1), bf16(c["q"]).reshape(T, -1))
    assert torch.equal(k.reshape(T, -1), bf16(c["k"]).reshape(T, -1))
    assert torch.equal(v.reshape(T, -1), qkv[:, (H + KVH) * 128:])
