"""The scratch cache layout of the non-causal (encoder) attention path, built with
tensor ops, against a per-sequence loop restatement of the same layout."""
import pytest
import torch


def _loop_layout(qsl, bs):
    S = len(qsl) - 1
    lens = [qsl[s + 1] - qsl[s] for s in range(S)]
    nblk = [(n + bs - 1) // bs for n in lens]
    width = max(max(nblk, default=1), 1)
    bt = torch.full((S, width), -1, dtype=torch.int32)
    slots, tok, pos, at = [], [], [], 0
    for s in range(S):
        bt[s, :nblk[s]] = torch.arange(at, at + nblk[s], dtype=torch.int32)
        slots += [at * bs + i for i in range(lens[s])]
        tok += [s] * lens[s]
        pos += [lens[s] - 1] * lens[s]
        at += nblk[s]
    return bt, slots, tok, pos, max(sum(nblk), 1)


@pytest.mark.parametrize("lens", [[5], [16, 1, 33, 0, 17], [1, 1, 1], [64, 15, 16, 100], []])
def test_encoder_layout_matches_loop(lens):
    from vllm_apple_b200.attention import encoder_layout
    qsl = [0]
    for n in lens:
        qsl.append(qsl[-1] + n)
    bt, slots, tok, pos, total = encoder_layout(qsl, 16)
    ebt, eslots, etok, epos, etotal = _loop_layout(qsl, 16)
    assert torch.equal(bt, ebt)
    assert slots.tolist() == eslots and slots.dtype == torch.int64
    assert tok.tolist() == etok and tok.dtype == torch.int32
    assert pos.tolist() == epos and pos.dtype == torch.int32
    assert total == etotal
