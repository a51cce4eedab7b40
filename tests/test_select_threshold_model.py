"""CPU model of the candidate selection in the per-phase select kernel (k_sa_fwd4, murm_ops.cu),
checked against the stable-sort top 7 (ties to the lowest slot) on random, tied and masked rows.

The kernel gives lane l (of 32) the slots l + 32 j, j < 8, turns each score into an order-keeping
32-bit key (0: no slot, -inf: masked), takes thr = the 7th largest of the 32 lanes' maximum keys
(ties counted), keeps only keys >= thr and ranks those by counting, in the order (key descending,
slot ascending); more than 32 candidates take a lane-list merge that ranks every key. This model
restates those steps with numpy and asserts that they return exactly the reference rule's picks.
"""
import numpy as np
import pytest

TOP_K = 7


def rank_keys(scores: np.ndarray) -> np.ndarray:
    """Order-keeping uint32 keys of fp32 scores (larger score -> larger key); -inf stays above 0."""
    bits = scores.astype(np.float32).view(np.uint32)
    neg = (bits & 0x80000000) != 0
    return np.where(neg, ~bits, bits | 0x80000000).astype(np.uint32)


def kernel_picks(scores: np.ndarray) -> np.ndarray:
    """The kernel's steps for one row of M <= 256 scores (masked entries already -inf)."""
    M = scores.shape[0]
    keys = np.zeros(256, dtype=np.uint32)
    keys[:M] = rank_keys(scores)
    lanes = keys.reshape(8, 32).T                      # lanes[l, j] = key of slot l + 32 j
    lane_max = lanes.max(axis=1)
    v, cnt, thr = lane_max.copy(), 0, 0
    for _ in range(TOP_K):                             # the 7th largest lane maximum, ties counted
        if cnt >= TOP_K:
            break
        best = v.max()
        thr = best
        cnt += int((v == best).sum())
        v[v == best] = 0
    slots = np.arange(256)
    cand = (keys != 0) & (keys >= thr)
    if cand.sum() > 32:                                # the lane-list merge ranks every key
        cand = keys != 0
    ck, cs = keys[cand].astype(np.int64), slots[cand]
    rank = np.array([((ck > k) | ((ck == k) & (cs < s))).sum() for k, s in zip(ck, cs)])
    out = np.empty(TOP_K, dtype=np.int64)
    for k, s, r in zip(ck, cs, rank):
        if r < TOP_K:
            out[r] = s
    return out


def reference_picks(scores: np.ndarray) -> np.ndarray:
    return np.argsort(-scores.astype(np.float64), kind="stable")[:TOP_K]


@pytest.mark.parametrize("M", [7, 40, 100, 255, 256])
def test_random_rows(M):
    rng = np.random.default_rng(M)
    for _ in range(200):
        s = rng.standard_normal(M).astype(np.float32)
        assert np.array_equal(kernel_picks(s), reference_picks(s))


def test_ties_and_repeated_keys():
    rng = np.random.default_rng(1)
    for _ in range(200):
        base = rng.standard_normal(int(rng.integers(2, 40))).astype(np.float32)
        s = base[rng.integers(0, base.size, 256)]      # many exact ties, across and within lanes
        assert np.array_equal(kernel_picks(s), reference_picks(s))


def test_masked_rows():
    rng = np.random.default_rng(2)
    for keep in (0, 1, 3, 6, 7, 8, 20):
        for _ in range(50):
            s = np.full(256, -np.inf, dtype=np.float32)
            idx = rng.choice(256, keep, replace=False)
            s[idx] = rng.standard_normal(keep).astype(np.float32)
            assert np.array_equal(kernel_picks(s), reference_picks(s))   # masked picks: lowest slots


def test_threshold_bounds_the_seventh_key():
    rng = np.random.default_rng(3)
    for _ in range(500):
        s = rng.standard_normal(256).astype(np.float32) * rng.uniform(0.01, 100)
        keys = rank_keys(s)
        lane_max = keys.reshape(8, 32).max(axis=0)
        thr = np.sort(lane_max)[-TOP_K]
        assert np.sort(keys)[-TOP_K] >= thr
