"""Cross-check of the router semantics against an independent implementation.

The oracle defines routing as: bf16 router logits, top-k of them (ties to the
lower expert index), weights = fp32 softmax over all experts gathered at the
selection and renormalised.  The installed Transformers Qwen3.5-MoE router
(``Qwen3_5MoeTopKRouter``: softmax in fp32, ``torch.topk``, divide by the
selected sum) is run here on the oracle's own bf16 logits: an identity router
weight makes its linear layer return those logits exactly, so every later
step is Transformers' code.  It must select the same experts in the same
order, and give the same renormalised weights to fp32 rounding.

Exact ties at the k-th place are resolved by the tie rule, which Transformers
leaves to torch.topk; where one occurs the test checks that the tied
experts have the same logit and that the oracle took the lower index.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from runnel_b200 import inputs

transformers = pytest.importorskip("transformers")
qmoe = pytest.importorskip("transformers.models.qwen3_5_moe.modeling_qwen3_5_moe")


class _Cfg:
    def __init__(self, E, k):
        self.num_experts = E
        self.num_experts_per_tok = k
        self.hidden_size = E


@pytest.mark.parametrize("bits,seed,T,skew", [(8, 0, 64, None), (4, 1, 64, None), (8, 2, 48, "zipf"),
                                             (8, 4, 48, "adversarial")])
def test_transformers_router_on_oracle_logits(bits, seed, T, skew):
    blk = inputs.make_block(bits, seed=seed, T=T, H=2048, I=256, E=256, skew=skew)
    w = oracle.BlockWeights(bits=bits, group=64, **blk.weight_fields())
    logits, inds, scores, _ = oracle.router(w, blk.x, k=8)
    router = qmoe.Qwen3_5MoeTopKRouter(_Cfg(256, 8))
    with torch.no_grad():
        router.weight.copy_(torch.eye(256))
        _, t_scores, t_inds = router(torch.from_numpy(logits))
    t_inds = t_inds.numpy()
    t_scores = t_scores.numpy()
    checked = 0
    for t in range(T):
        order = np.argsort(-logits[t], kind="stable")  # lower index first among equals
        kth, nxt = logits[t, order[7]], logits[t, order[8]]
        if kth != nxt:
            # no tie at the boundary: same experts, same order (descending logit)
            np.testing.assert_array_equal(np.sort(t_inds[t]), np.sort(inds[t]))
            # within equal logits the order may differ; compare logit sequences
            np.testing.assert_array_equal(logits[t, t_inds[t]], logits[t, inds[t]])
            np.testing.assert_allclose(t_scores[t][np.argsort(t_inds[t])], scores[t][np.argsort(inds[t])],
                                       rtol=2e-6, atol=0)
            checked += 1
        else:
            # tie at the k-th place: the same multiset of logits, the oracle
            # taking the lowest indices of the tied value
            np.testing.assert_array_equal(np.sort(logits[t, t_inds[t]]), np.sort(logits[t, inds[t]]))
            tied = np.flatnonzero(logits[t] == kth)
            chosen = sorted(set(inds[t].tolist()) & set(tied.tolist()))
            assert chosen == sorted(tied.tolist())[:len(chosen)]
    assert checked >= T // 2
    # the oracle's slot order is descending logit, ties to the lower index
    for t in range(T):
        lv = logits[t, inds[t]]
        assert np.all(lv[:-1] >= lv[1:])
