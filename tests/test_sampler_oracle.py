"""The oracle of the reference's vLLM sampler kernels
(csrc/aten/vllm_kernels/min_p.cpp, logprob.cpp) on small known answers."""

import numpy as np

import oracle


def test_min_p_known_answers():
    x = np.array([[1.0, 3.0, 2.0, -1.0], [0.0, 0.0, 5.0, 4.9]], dtype=np.float32)
    mp = np.array([0.0, 0.5, 1.0], dtype=np.float32)
    # row 0 -> request 0 (p = 0): unchanged; row 1 -> request 2 (p = 1): only the maximum survives
    out = oracle.vllm_min_p(x, np.array([0, 2]), mp, 4)
    assert np.array_equal(out[0], x[0])
    assert out[1].tolist() == [-np.inf, -np.inf, 5.0, -np.inf]
    # p = 0.5: threshold 3 + log(0.5) = 2.3069: keeps 3 only
    out = oracle.vllm_min_p(x[:1], np.array([1]), mp, 4)
    assert out[0].tolist() == [-np.inf, 3.0, -np.inf, -np.inf]


def test_log_softmax_and_ranks_known_answers():
    x = np.array([[0.0, np.log(3.0), 0.0, 0.0]], dtype=np.float32)  # softmax = [1/6, 1/2, 1/6, 1/6]
    lp = oracle.vllm_topk_log_softmax(x, np.array([[1, 0, 99, -5]]), 4)
    np.testing.assert_allclose(lp[0], np.log([0.5, 1 / 6, 1 / 6, 1 / 6]), rtol=1e-6)  # 99 and -5 clamp
    assert oracle.vllm_ranks(x, np.array([1]), 4).tolist() == [1]
    assert oracle.vllm_ranks(x, np.array([0]), 4).tolist() == [4]  # ties count


def test_penalties_known_answers():
    """penalties.cpp:14-84 by hand: vocab 4, rep 2, freq 0.5, pres 0.25; token 0
    in the prompt, token 2 generated three times."""
    lg = np.array([[2.0, -2.0, 1.0, 4.0]], dtype=np.float32)
    pbm = np.array([[0b0001]], dtype=np.int32)
    obc = np.array([[0, 0, 3, 0]], dtype=np.int32)
    out = oracle.vllm_penalties(lg, np.array([0]), np.array([1]), np.array([0]), np.array([2.0]),
                                np.array([0.5]), np.array([0.25]), pbm, obc, 4, 0)
    # 2 / 2 = 1; -2 untouched; 1 / 2 - 0.5 * 3 - 0.25 = -1.25; 4 untouched
    assert out.tolist() == [[1.0, -2.0, -1.25, 4.0]]
    # a negative logit in the prompt is multiplied: -2 * 2
    out = oracle.vllm_penalties(lg, np.array([0]), np.array([1]), np.array([0]), np.array([2.0]),
                                np.array([0.0]), np.array([0.0]), np.array([[0b0010]], dtype=np.int32),
                                np.zeros((1, 4), np.int32), 4, 0)
    assert out.tolist() == [[2.0, -4.0, 1.0, 4.0]]
    # neutral penalties leave the row, whatever the counts
    out = oracle.vllm_penalties(lg, np.array([0]), np.array([1]), np.array([0]), np.array([1.0]),
                                np.array([0.0]), np.array([0.0]), pbm, obc, 4, 0)
    assert np.array_equal(out, lg)


def test_penalties_draft_tokens():
    """Row t at local position pos counts the drafts token_ids[t-pos+1 .. t],
    and only with max_spec_len > 0."""
    lg = np.ones((3, 4), dtype=np.float32)
    args = (np.array([0, 0, 0]), np.array([9, 3, 2]), np.array([0, 1, 2]), np.array([1.0]), np.array([1.0]),
            np.array([0.0]), np.zeros((1, 1), np.int32), np.zeros((1, 4), np.int32), 4)
    out = oracle.vllm_penalties(lg, *args, 2)
    assert out.tolist() == [[1, 1, 1, 1], [1, 1, 1, 0], [1, 1, 0, 0]]
    assert np.array_equal(oracle.vllm_penalties(lg, *args, 0), lg)


def test_bincount_known_answers():
    tids = np.array([[0, 0, 0, 0], [33, 1, 1, 5]])
    pbm, obc = oracle.vllm_bincount(np.array([1]), tids, np.array([0, 2]), np.array([0, 4]),
                                    np.zeros((2, 2), np.int32), np.zeros((2, 40), np.int32))
    assert pbm.tolist() == [[0, 0], [2, 2]]  # 33 -> word 1 bit 1; 1 -> word 0 bit 1
    assert obc[1, :6].tolist() == [0, 1, 0, 0, 0, 1] and obc[0].sum() == 0
    # bit 31 sets the sign bit; tokens past the mask or the vocabulary are skipped
    pbm, obc = oracle.vllm_bincount(np.array([0]), np.array([[31, 64, 40, 7]]), np.array([2]), np.array([4]),
                                    np.zeros((1, 2), np.int32), np.zeros((1, 16), np.int32))
    assert pbm.tolist() == [[-(2 ** 31), 0]]
    assert obc[0].tolist() == [0] * 7 + [1] + [0] * 8


def test_bias_known_answers():
    """logit_bias.cpp:15-96 by hand: allowed ids [3, 9 -> clamped to 3], bias
    +0.5 and +0.25 on id 3 (in order) and +7 on a masked id, stop id 1 while
    pos 1 < min_len 5."""
    lg = np.array([[1.0, 2.0, 3.0, 4.0]], dtype=np.float32)
    args = (4, np.array([0]), np.array([2]), np.array([[3, 9]]), np.array([3]), np.array([[3, 3, 0]]),
            np.array([[0.5, 0.25, 7.0]], dtype=np.float32))
    out = oracle.vllm_bias(lg, *args, np.array([1]), np.array([5]), np.array([1]), np.array([[1]]))
    assert out.tolist() == [[-np.inf, -np.inf, -np.inf, 4.75]]
    # no allowed list, pos past min_len: only the biases
    out = oracle.vllm_bias(lg, 4, np.array([0]), np.array([0]), np.array([[0, 0]]), np.array([2]),
                           np.array([[2, -1, 0]]), np.array([[0.5, 9.0, 0.0]], dtype=np.float32),
                           np.array([5]), np.array([5]), np.array([1]), np.array([[1]]))
    assert out.tolist() == [[1.0, 2.0, 3.5, 4.0]]


def test_bad_words_known_answers():
    """bad_words.cpp:13-82 by hand: output so far [7, 8], bad words [8, 3]
    (prefix 8 ends the output: bans 3), [7, 9, 4] (prefix 7 9 does not: 4
    stays) and [5] (no prefix: always bans 5)."""
    lg = np.zeros((1, 10), dtype=np.float32)
    ids = np.array([[8, 3, 7, 9, 4, 5]])
    off = np.array([[0, 2, 5, 6]])
    tids = np.array([[1, 2, 7, 8, 0]])  # prompt [1, 2], output [7, 8]
    out = oracle.vllm_bad_words(lg, np.array([0]), ids, off, np.array([3]), tids, np.array([2]), np.array([4]),
                                np.array([0]), np.array([0]))
    assert np.isneginf(out[0]).nonzero()[0].tolist() == [3, 5]
    # two rows of one request: row 1 (pos 1) sees the output then the draft
    # input_ids[0] = 9, so [9, 4] bans 4 there and [8, 3] bans 3 on row 0
    out = oracle.vllm_bad_words(np.zeros((2, 10), np.float32), np.array([0, 0]), np.array([[9, 4, 8, 3]]),
                                np.array([[0, 2, 4]]), np.array([2]), tids, np.array([2]), np.array([4]),
                                np.array([9, 6]), np.array([0, 1]))
    assert np.isneginf(out[0]).nonzero()[0].tolist() == [3]  # row 0 ends in 8
    assert np.isneginf(out[1]).nonzero()[0].tolist() == [4]  # row 1 ends in the draft 9
