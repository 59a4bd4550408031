"""The oracle of the MoE dispatch step (moe_align_block_size) on the CPU:
pinned to the worked example of vLLM's documentation of the op
(vllm/model_executor/layers/fused_moe/moe_align_block_size.py:59-72:
topk_ids [[2,3,4],[1,2,4],[1,3,4],[1,2,3]], block_size 4, with expert ids
1..4, i.e. 5 experts of which expert 0 is empty), and checked for the
properties the contract states on random inputs."""

import numpy as np
import pytest

import oracle


def test_documented_example():
    ids = np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]])
    s, e, n = oracle.moe_align_block_size(ids, 5, 4)
    assert n == 16
    assert s[:n].tolist() == [3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12]
    assert e[: n // 4].tolist() == [1, 2, 3, 4]
    assert (s[n:] == 12).all() and (e[n // 4:] == -1).all()


@pytest.mark.parametrize("T,K,E,bs", [(1, 8, 256, 16), (33, 6, 160, 64), (500, 8, 256, 1), (64, 2, 8, 128),
                                      (3, 4, 1024, 32)])
def test_contract_properties(T, K, E, bs):
    rng = np.random.default_rng(T * 7 + E)
    ids = rng.integers(0, E, size=(T, K))
    s, e, n = oracle.moe_align_block_size(ids, E, bs)
    numel = T * K
    flat = ids.reshape(-1)
    assert n % bs == 0 and len(s) == min(numel + E * (bs - 1), numel * bs)
    real = s[s < numel]
    assert sorted(real.tolist()) == list(range(numel))  # every entry exactly once
    for b in range(n // bs):
        blk = s[b * bs:(b + 1) * bs]
        toks = blk[blk < numel]
        assert (flat[toks] == e[b]).all()  # a block holds one expert's entries
        assert (np.diff(toks) > 0).all()  # ascending within the block
    runs = [e[b] for b in range(n // bs)]
    assert runs == sorted(runs)  # experts in order


def test_out_of_range_entries_are_left_out():
    ids = np.array([[0, 5, -1], [1, 1, 9]])
    s, e, n = oracle.moe_align_block_size(ids, 4, 2)
    assert n == 4 and s[:n].tolist() == [0, 6, 3, 4]
