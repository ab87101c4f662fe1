"""Host model (numpy) of the decode kernel's lazy-rescale online softmax, in both of its forms, against exact
attention: the plain form (scores scaled, the vote compares them with m + 2^8) and the speculative-weights form of the
48-row variant (weights 2^(s * scale - m) first, a thread votes when its weights add up to 2^8, the exact path then
takes the tile maxima and the weights again, and O accumulates across tiles with an alpha correction).  It checks the
invariant both forms rely on -- no weight above 2^8, so bf16 P and FP32 sums stay exact enough -- and that the result
is the softmax of the exact path.  The kernels themselves are checked on the GPU against the oracle
(tests/test_gpu_decode.py); this pins the schedule they implement."""
import numpy as np
import pytest

TILE = 128
THRESH = 8.0


def bf16(x):
    """Round float32 to bfloat16 (nearest even) and back."""
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def exact(q, k, v, scale, lens_visible):
    """float64 attention; row r sees keys [0, lens_visible[r])."""
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    for r, n in enumerate(lens_visible):
        s[r, n:] = -np.inf
    p = np.exp(s - s.max(1, keepdims=True))
    return (p / p.sum(1, keepdims=True)) @ v.astype(np.float64)


def online(q, k, v, scale, lens_visible, speculative, group_rows=24):
    """One segment through the kernel's schedule: tiles of 128 keys, row groups of `group_rows` rows (a group's vote
    spans its 128 token-threads, each thread holding one key's scores for the group's rows)."""
    R, L = q.shape[0], k.shape[0]
    sl2 = np.float32(scale * np.log2(np.e))
    m = np.full(R, -np.inf, np.float32)
    l = np.zeros(R, np.float32)
    o = np.zeros((R, v.shape[1]), np.float32)
    stats = {"max_weight": 0.0, "rescales": 0, "tiles": 0}
    for t0 in range(0, L, TILE):
        kt, vt = k[t0:t0 + TILE], v[t0:t0 + TILE]
        s = (q @ kt.T).astype(np.float32)                     # [R, tokens], unscaled
        tok = np.arange(t0, t0 + kt.shape[0])
        s = np.where(tok[None, :] < np.asarray(lens_visible)[:, None], s, -np.inf).astype(np.float32)
        first = t0 == 0
        stats["tiles"] += 1
        for g0 in range(0, R, group_rows):
            rows = slice(g0, min(R, g0 + group_rows))
            sg, mg = s[rows], m[rows]
            negm = np.where(np.isneginf(mg), 0, -mg).astype(np.float32)
            if speculative:
                need = first
                if not first:
                    p = np.exp2(sg * sl2 + negm[:, None]).astype(np.float32)
                    need = bool((p.sum(0) >= 2 ** THRESH).any())   # per token-thread sums over the group's rows
            else:
                sc = sg * sl2
                need = first or bool((sc > mg[:, None] + THRESH).any())
            alpha = np.ones_like(mg)
            if need:
                stats["rescales"] += 1
                tm = sg.max(1) * sl2
                mn = np.where(first | (tm > mg + THRESH), np.maximum(mg, tm), mg).astype(np.float32)
                alpha = np.where(np.isneginf(mg) | (mn == mg), 1, np.exp2(mg - mn)).astype(np.float32)
                m[rows] = mn
                negm = np.where(np.isneginf(mn), 0, -mn).astype(np.float32)
            p = np.exp2(sg * sl2 + negm[:, None]).astype(np.float32)
            stats["max_weight"] = max(stats["max_weight"], float(p.max(initial=0)))
            l[rows] = l[rows] * alpha + p.sum(1)
            # O: scaled by alpha before this tile's PV product adds on (in TMEM for the speculative form, in
            # registers for the plain one: the same arithmetic); P goes to the tensor core as bf16
            o[rows] = o[rows] * alpha[:, None] + bf16(p) @ vt
    return o / np.where(l > 0, l, 1)[:, None], stats


def segment(seed, L, n, G=4, rising=0.0):
    rng = np.random.default_rng(seed)
    q = bf16(rng.standard_normal((n * G, 128)).astype(np.float32))
    k = bf16(rng.standard_normal((L, 128)).astype(np.float32))
    v = bf16(rng.standard_normal((L, 128)).astype(np.float32))
    if rising:
        q[:, 0] = 4.0
        k[:, 0] += bf16(rising * np.arange(L, dtype=np.float32))
    lens = [L - n + 1 + r // G for r in range(n * G)]   # row r = i * G + h sees keys <= L - n + i
    return q, k, v, lens


@pytest.mark.parametrize("speculative", [False, True])
@pytest.mark.parametrize("L,n,rising", [(1000, 9, 0.0), (2047, 12, 0.0), (700, 9, 0.3), (129, 9, 0.0), (12, 12, 0.0)])
def test_schedule_matches_exact_softmax_and_bounds_weights(speculative, L, n, rising):
    q, k, v, lens = segment(L + n, L, n, rising=rising)
    scale = 128 ** -0.5
    got, st = online(q, k, v, scale, lens, speculative)
    ref = exact(q, k, v, scale, lens)
    assert st["max_weight"] <= 2 ** THRESH
    err = np.abs(got - ref)
    assert (err <= 1e-2 + 1e-2 * np.abs(ref)).all(), float(err.max())
    groups = -(-n * 4 // 24)
    if rising:
        assert st["rescales"] == st["tiles"] * groups   # every tile moves the maxima past the threshold
    else:
        assert st["rescales"] == groups                  # only the first tile of the segment takes the exact path


def test_speculative_vote_catches_a_late_large_score():
    """A single key far above the running maxima late in the segment: the weight sum of the thread that holds it
    passes 2^8, so the exact path runs and no weight exceeds 2^8."""
    q, k, v, lens = segment(7, 900, 9)
    k[777] = bf16(q[0] * 3.0)   # row 0 scores ~3 * |q_0|^2 / sqrt(128) on key 777, far above the rest
    scale = 128 ** -0.5
    got, st = online(q, k, v, scale, lens, speculative=True)
    assert st["rescales"] > 2 and st["max_weight"] <= 2 ** THRESH
    ref = exact(q, k, v, scale, lens)
    assert np.abs(got - ref).max() <= 1e-2 + 1e-2 * np.abs(ref).max()
