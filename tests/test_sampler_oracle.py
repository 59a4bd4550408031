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
