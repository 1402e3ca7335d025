"""The reference's custom op pseudobrain::gated_delta_chunk (gated_deltanet.py:200-227) as this
package registers it: the schema and the fake (meta) shapes on any host, and -- where the
reference itself is importable -- this package's CUDA kernel attached to the reference's own op.
Compute parity is a GPU test (tests/test_fla_op_gpu.py)."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import gdn as ogdn
from tests.conftest import ROOT

REFERENCE = "/root/reference"


def _run(code: str) -> str:
    env = dict(os.environ, PYTHONPATH=ROOT)
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, check=True,
                          timeout=600).stdout


def test_op_defined_with_reference_schema_and_fake_shapes():
    out = _run("""
import torch
import pseudobrain_b200.fla_op as f
assert f.DEFINED_HERE
schema = str(torch.ops.pseudobrain.gated_delta_chunk.default._schema)
print(schema)
q = torch.empty(2, 100, 4, 128, device="meta", dtype=torch.bfloat16)
v = torch.empty(2, 100, 4, 128, device="meta", dtype=torch.bfloat16)
g = torch.empty(2, 100, 4, device="meta")
h0 = torch.empty(2, 4, 128, 128, device="meta")
o, s, gc, a = torch.ops.pseudobrain.gated_delta_chunk(q, q, v, g, g.to(torch.bfloat16), h0, 0.1)
print(tuple(o.shape), o.dtype, tuple(s.shape), s.dtype, tuple(gc.shape), gc.dtype, tuple(a.shape), a.dtype)
try:
    torch.ops.pseudobrain.gated_delta_chunk(*(torch.zeros(x.shape, dtype=x.dtype) for x in (q, q, v, g)),
                                            torch.zeros(2, 100, 4), torch.zeros(2, 4, 128, 128), 0.1)
    print("cpu ran")
except RuntimeError:
    print("cpu raises")
""")
    lines = out.strip().splitlines()
    assert "gated_delta_chunk(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor h0, float scale)" in lines[0]
    assert lines[1] == ("(2, 100, 4, 128) torch.bfloat16 (2, 4, 128, 128) torch.float32 (2, 100, 4) torch.float32 "
                        "(2, 100, 4, 64) torch.bfloat16")
    assert lines[2] == "cpu raises"


@pytest.mark.skipif(not os.path.isdir(os.path.join(REFERENCE, "pseudobrain")), reason="reference not present")
def test_kernel_attached_to_the_reference_op():
    out = _run(f"""
import sys, torch
sys.path.insert(0, {REFERENCE!r})
import pseudobrain.gated_deltanet as ref
import pseudobrain_b200.fla_op as f
assert not f.DEFINED_HERE
print(torch._C._dispatch_has_kernel_for_dispatch_key("pseudobrain::gated_delta_chunk", "CUDA"))
""")
    assert out.strip().splitlines()[-1] == "True"


def test_chunk_aux_oracle_matches_chunked_algorithm():
    """oracle.gdn.chunk_aux's T reproduces the chunked algorithm's U' = T diag(beta) V: the
    first chunk's outputs from a zero state equal (Q K^T o D) U' (delta_rule_chunked)."""
    from tests.inputs import gdn_inputs
    inp = gdn_inputs(31, 1, 64, 1, 1)
    gc, ta = ogdn.chunk_aux(inp["k"], inp["g"], inp["beta"])
    assert np.allclose(gc[0, :, 0], np.cumsum(inp["g"][0, :, 0], dtype=np.float32), rtol=1e-6)
    q, k, v, beta = inp["q"][0, :, 0], inp["k"][0, :, 0], inp["v"][0, :, 0], inp["beta"][0, :, 0]
    c = gc[0, :, 0].astype(np.float64)
    d = np.tril(np.exp(c[:, None] - c[None, :]))
    uprime = ta[0, :, 0].astype(np.float64) @ (v * beta[:, None])
    o = ((q * inp["scale"]) @ k.T * d) @ uprime
    ro, _ = ogdn.delta_rule_chunked(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["scale"], inp["h0"])
    assert ogdn.rel_err(o, ro[0, :, 0]) < 1e-5
