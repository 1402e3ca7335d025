"""The numpy restatement of vLLM's decode ops (oracle/vllm_decode.py) agrees with the oracle
pinned to the reference's golden outputs: the per-step recurrence (gated_deltanet.py:93-107)
in vLLM's [V, K] pool layout, the gating of gated_deltanet.py:427-429 and the 'hf' q/k norm."""
from __future__ import annotations

import numpy as np

from oracle import gdn as ogdn
from oracle import vllm_decode as ovd
from tests.inputs import gdn_inputs


def test_recurrent_equals_sequential_rule_in_pool_layout():
    inp = gdn_inputs(21, 3, 4, 2, 4, state_std=0.05)
    q, k = inp["q"], inp["k"]
    hv = 4
    pool = np.ascontiguousarray(inp["h0"].transpose(0, 1, 3, 2))  # [B, HV, V, K]
    o, new = ovd.recurrent(q, k, inp["v"], inp["g"], inp["beta"], inp["scale"], pool)
    ro, rs = ogdn.delta_rule_sequential(ogdn.expand_key_heads(q, hv), ogdn.expand_key_heads(k, hv), inp["v"],
                                        inp["g"], inp["beta"], inp["scale"], inp["h0"])
    assert ogdn.rel_err(o, ro) < 1e-5
    assert ogdn.rel_err(new, rs.transpose(0, 1, 3, 2)) < 1e-5


def test_gating_and_norm_match_layer_oracle():
    rng = np.random.default_rng(3)
    a, b = rng.standard_normal((5, 4)) * 3, rng.standard_normal((5, 4))
    a_log, dt = rng.standard_normal(4), rng.standard_normal(4)
    g, beta = ovd.gating(a, b, a_log, dt)
    rg, rb = ogdn.gating(a, b, a_log, dt)
    assert np.allclose(g, rg, rtol=1e-6) and np.allclose(beta, rb, rtol=1e-6)
    x = rng.standard_normal((2, 3, 128))
    assert np.allclose(ovd._norm(x, 2), ogdn.l2_normalize(x, "hf", 1e-6), rtol=1e-6)
    assert np.allclose(ovd._norm(x, 1), ovd._norm(x, 2), rtol=1e-12)


def test_speculative_columns_and_null_slots():
    """Column t of a 2-D index row receives the state after token t; the initial state comes
    from column num_accepted - 1; null entries (<= 0) are neither read nor written."""
    inp = gdn_inputs(22, 1, 5, 1, 2, state_std=0.05)
    pool = np.stack([np.ascontiguousarray(inp["h0"][0].transpose(0, 2, 1))] * 8)
    idx = np.array([[3, 4, 0, 6, 7], [0, 0, 0, 0, 0]])
    cu = np.array([0, 5, 5])
    o, new = ovd.recurrent(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["scale"], pool, cu_seqlens=cu,
                           indices=idx, num_accepted=np.array([2, 1]))
    # from column 1 (slot 4): the same as starting from that state
    o1, s_seq = ogdn.delta_rule_sequential(ogdn.expand_key_heads(inp["q"], 2), ogdn.expand_key_heads(inp["k"], 2),
                                           inp["v"], inp["g"], inp["beta"], inp["scale"],
                                           pool[4][None].transpose(0, 1, 3, 2))
    assert ogdn.rel_err(o, o1) < 1e-5
    assert ogdn.rel_err(new[7], s_seq[0].transpose(0, 2, 1)) < 1e-5
    assert np.array_equal(new[0], pool[0]) and np.array_equal(new[5], pool[5])
