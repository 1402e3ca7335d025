"""GPU parity of pseudobrain::gated_delta_chunk (the reference's fla custom op, gated_deltanet.py:
200-227, on this package's kernels) against the oracle: o in q's dtype and the final state
(2e-2 for bf16 inputs, 1e-4 for fp32), the chunk-local cumulative g (fp32 sums in another
order: 1e-5) and the WY inverse T (bf16 storage for bf16 inputs: 1e-2; fp32 inputs: 1e-4),
over ragged lengths and both paths (tensor-core for bf16, exact fp32 otherwise)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from tests.inputs import gdn_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bf16,batch,length,hv", [(True, 2, 300, 4), (True, 1, 64, 2), (True, 1, 37, 2),
                                                  (False, 2, 150, 2)])
def test_gated_delta_chunk_matches_oracle(cuda_device, bf16, batch, length, hv):
    import pseudobrain_b200.fla_op as f
    inp = gdn_inputs(40 + length, batch, length, hv, hv, bf16=bf16, state_std=0.02)
    dt = torch.bfloat16 if bf16 else torch.float32
    q, k, v, beta = (torch.from_numpy(inp[n]).to(cuda_device, dt) for n in ("q", "k", "v", "beta"))
    g = torch.from_numpy(inp["g"]).to(cuda_device)
    h0 = torch.from_numpy(inp["h0"]).to(cuda_device)
    o, final, gc, a = torch.ops.pseudobrain.gated_delta_chunk(q, k, v, g, beta, h0, inp["scale"])
    assert o.dtype == dt and final.dtype == torch.float32 and gc.dtype == torch.float32 and a.dtype == dt
    assert a.shape == (batch, length, hv, 64)
    ro, rs = ogdn.delta_rule_chunked(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["scale"], inp["h0"])
    rgc, ra = ogdn.chunk_aux(inp["k"], inp["g"], inp["beta"])
    tol = 2e-2 if bf16 else 1e-4
    assert ogdn.rel_err(o.float().cpu().numpy(), ro) < tol
    assert ogdn.rel_err(final.cpu().numpy(), rs) < tol
    assert np.allclose(gc.cpu().numpy(), rgc, rtol=1e-5, atol=1e-5)
    assert ogdn.rel_err(a.float().cpu().numpy(), ra) < (1e-2 if bf16 else 1e-4)
    # the reference's fla route (delta_rule_fla) through the op
    of, sf = f.delta_rule_fla(q, k, v, g, beta, inp["scale"], h0)
    assert of.dtype == torch.float32 and ogdn.rel_err(of.cpu().numpy(), ro) < tol
