"""Helpers shared by test modules: re-exports of the conftest helpers and the
MoE routing/layer checks used by several GPU tests."""
import numpy as np

import oracle
from conftest import from_bits, rel_err, to_bits  # noqa: F401


def check_moe_routing_and_layer(layer, x_bits, w13_bits, w2_bits, wr_bits, out, k,
                                record=None):
    """The MoE checks shared by the layer tests:
    * routing bit-exact given the GPU's fp32 logits: the oracle's top-k on
      those logits gives the GPU's indices exactly (and its softmax weights
      within 1e-5 relative: the GPU's exp is not the host's);
    * the GPU logits within 1e-5 (relative L2) of the oracle's own;
    * tokens whose top-k from the oracle's own logits differs from the GPU's
      are counted (near ties); each must be a tie to within 1e-4 in the
      oracle's logits;
    * the whole layer output (every token) within 1e-2 of the oracle run on
      the GPU's routing.
    Returns the near-tie count."""
    rt = layer.last_routing
    g_logits = rt.logits.float().cpu().numpy()
    g_idx = rt.topk_idx.cpu().numpy()
    g_w = rt.topk_w.cpu().numpy()
    o_idx, o_w = oracle.moe_topk(g_logits, k)
    assert np.array_equal(o_idx, g_idx)
    np.testing.assert_allclose(g_w, o_w, rtol=1e-5, atol=1e-7)   # probabilities
    ref_logits = oracle.gemm(x_bits, wr_bits, b_layout="nk", out_f32=True)
    assert rel_err(g_logits, ref_logits) < 1e-5
    r_idx, _ = oracle.moe_topk(ref_logits, k)
    flips = ~(r_idx == g_idx).all(axis=1)
    gaps = oracle.topk_gap(ref_logits, k)
    n_ties = int(flips.sum())
    assert (gaps[flips] < 1e-4).all(), gaps[flips]
    if record is not None:
        record("near_tie_tokens", n_ties)
    print(f"near-tie tokens (top-k flips between GPU and oracle logits): {n_ties} "
          f"of {len(g_idx)}")
    ref = oracle.moe_layer_given_routing(x_bits, w13_bits, w2_bits, g_idx, g_w)
    got = oracle.bf16_to_f32(to_bits(out))
    assert np.isfinite(got).all()
    assert rel_err(got, oracle.bf16_to_f32(ref)) < 1e-2
    return n_ties
