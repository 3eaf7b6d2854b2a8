"""Top-k oracle pinned to the reference's own selection (CPU).

``oracle.topk`` must give, value for value, what the reference kernel's two-stage
insertion lists give (vllm_apple/engine/ops/topk.py:80-226), and what the
reference's own numpy check sorts to (argsort of the row, largest k;
docs/debug-archive/test_topk_standalone.py:53-66) on rows without NaN / -inf.
"""
import numpy as np
import pytest

from oracle import paged_attention as ref


def _rows(seed, T, V, special=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, V)).astype(np.float16)
    if special:
        x[0, rng.integers(0, V, 5)] = np.nan
        x[0, rng.integers(0, V, 5)] = -np.inf
        x[0, rng.integers(0, V, 2)] = np.inf
        x[min(1, T - 1), :] = np.float16(0.5)          # all ties
        x[min(2, T - 1), : V // 2] = -np.inf           # short of valid logits
        x[min(2, T - 1), V // 2:] = np.nan
    return x


@pytest.mark.parametrize("T,V,k", [(2, 257, 8), (3, 300, 50), (1, 64, 1), (2, 40, 64)])
@pytest.mark.parametrize("special", [False, True])
def test_oracle_matches_insertion_lists(T, V, k, special):
    x = _rows(T * V + k, T, V, special)
    i, v = ref.topk(x, k)
    ri, rv = ref.topk_insertion_lists(x, k)
    np.testing.assert_array_equal(v.astype(np.float32), rv.astype(np.float32))
    # wherever the reference's value is unique in the row the index is the same
    for t in range(T):
        for j in range(k):
            if ri[t, j] < 0:
                assert i[t, j] == -1
            elif np.sum(x[t] == x[t, ri[t, j]]) == 1:
                assert i[t, j] == ri[t, j]


@pytest.mark.parametrize("T,V,k", [(4, 1000, 50), (2, 32000, 8), (1, 151936, 100)])
def test_oracle_matches_argsort_values(T, V, k):
    x = _rows(V + k, T, V)
    i, v = ref.topk(x, k)
    for t in range(T):
        top = np.argsort(x[t].astype(np.float32))[-k:][::-1]
        np.testing.assert_array_equal(v[t], x[t, top])
        np.testing.assert_array_equal(x[t, i[t]], v[t])
    # ties ordered by index: within equal values the indices increase
    for t in range(T):
        same = v[t, 1:] == v[t, :-1]
        assert np.all(i[t, 1:][same] > i[t, :-1][same])


def test_oracle_padding_and_specials():
    x = np.array([[np.nan, -np.inf, 1.0, np.inf, -0.0, 0.0]], dtype=np.float16)
    i, v = ref.topk(x, 6)
    assert i.tolist() == [[3, 2, 5, 4, -1, -1]]
    assert np.isinf(v[0, 4]) and v[0, 4] < 0 and np.isinf(v[0, 0]) and v[0, 0] > 0


@pytest.mark.parametrize("T,V,k", [(3, 32000, 50), (2, 151936, 40), (4, 5000, 1)])
def test_oracle_matches_reference_cpu_sampler_topk(T, V, k):
    """The reference's own CPU sampler takes top-k with ``torch.topk(req_logits, top_k)``
    (vllm_apple/v1/worker/apple_model_runner.py:1799-1804).  On rows of distinct finite
    values the selection is unique, so the oracle's indices and values must equal it."""
    import torch
    rng = np.random.default_rng(T + V + k)
    bits = np.arange(-30000, 30000, dtype=np.int32).astype(np.int16).view(np.float16)
    pool = np.unique(bits[np.isfinite(bits)].astype(np.float32)).astype(np.float16)
    x = np.stack([rng.permutation(pool)[:V] if V <= pool.size else
                  np.concatenate([rng.permutation(pool),
                                  np.full(V - pool.size, -np.inf, np.float16)])
                  for _ in range(T)])
    i, v = ref.topk(x, k)
    tv, ti = torch.topk(torch.from_numpy(x.astype(np.float32)), k, dim=1)
    np.testing.assert_array_equal(i, ti.numpy())
    np.testing.assert_array_equal(v.astype(np.float32), tv.numpy())
