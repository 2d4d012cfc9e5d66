"""GPU tests of the plugin runtime (gdn_state_codec.runtime) on the B200
kernels: slot encode from a vLLM-style provider-layout state cache,
reconstruction, boundary readout and a decode step, checked against the CPU
oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import _native, codec
from gdn_state_codec import runtime as runtime_mod
from gdn_state_codec.config import GdnStateCodecExperiment

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
HEADS = 32


def bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


def runtime(initializer="quant_only"):
    experiment = GdnStateCodecExperiment(_native.library_dir(), "shadow", initializer,
                                         0 if initializer == "quant_only" else 4, "vector")
    return runtime_mod.GdnStateCodecRuntime(experiment, "model.layers.0.linear_attn")


@pytest.fixture(scope="module")
def ssm_state():
    """vLLM ssm_state-like cache: [slots, heads, value, key] fp32."""
    return codec.synthesize_states(6, 1, HEADS, layout="provider", seed=11,
                                   device=DEV).reshape(6, HEADS, 128, 128)


def test_quant_only_slot_encode_matches_oracle(ssm_state):
    rt = runtime()
    slot = rt._slot(ssm_state, 4)
    assert rt._slot(ssm_state, 4) is slot  # cached per cache index
    torch.cuda.synchronize()
    host = ssm_state[4].cpu().numpy()
    z, c, b = oracle.quantize(host, "provider")
    assert np.array_equal(slot.residual.cpu().numpy(), z)
    assert np.array_equal(bits(slot.smoothing.cpu().numpy()), bits(c))
    assert np.array_equal(bits(slot.scales.cpu().numpy()), bits(b))
    assert slot.compensator_keys.dtype == torch.float16
    assert not slot.compensator_keys.any() and not slot.compensator_values.any()


def test_reconstruct_and_boundary_readout(ssm_state):
    rt = runtime()
    slot = rt._slot(ssm_state, 2)
    dense = rt.reconstruct(slot)                      # [H, key, value]
    q = codec.synthesize_queries(1, 1, HEADS, seed=3, device=DEV).reshape(HEADS, 128)
    out = rt.boundary_readout(slot, q)
    torch.cuda.synchronize()
    z = slot.residual.cpu().numpy()
    c, b = slot.smoothing.cpu().numpy(), slot.scales.cpu().numpy()
    zeros = np.zeros((HEADS, 128, 4), np.float32)
    want = oracle.dequantize(z, c, b, zeros, zeros, layout="provider").transpose(0, 2, 1)
    assert np.array_equal(bits(dense.cpu().numpy()), bits(want))
    want_out = oracle.project(z, c, b, q.float().cpu().numpy(), zeros, zeros, layout="provider")
    assert np.array_equal(bits(out.cpu().numpy()), bits(want_out))
    # the readout is the reconstruction times the query, within fp32 rounding
    ref = torch.einsum("hkv,hk->hv", dense.double(), q.double())
    np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), rtol=1e-4, atol=1e-5)
    # shadow check of a state against itself passes the gate
    assert rt.observe_shadow(dense, ssm_state[2].transpose(-2, -1)) < runtime_mod.SHADOW_RELATIVE_RMS_LIMIT


def test_exact_svd_slot_quantizes_the_residual_exactly(ssm_state):
    rt = runtime("exact_svd")
    dense = ssm_state[1].transpose(-2, -1).contiguous()   # capsule order
    slot = rt._encode_dense_boundary(dense, "exact_svd")
    left = slot.compensator_keys.float()
    torch.cuda.synchronize()
    assert left.abs().max() > 0
    # the int8 stage runs on dense - U S V^T; recompute that residual the same
    # way and check the native quantizer against the oracle on it
    u, s, vt = torch.linalg.svd(dense, full_matrices=False)
    right = vt[:, :4, :].transpose(-2, -1)       # the runtime's exact views and ops
    residual = dense - torch.bmm(u[:, :, :4] * s[:, None, :4], right.transpose(-2, -1))
    z, c, b = oracle.quantize(residual.cpu().numpy(), "capsule")
    assert np.array_equal(slot.residual.transpose(-2, -1).cpu().numpy(), z)
    assert np.array_equal(bits(slot.smoothing.cpu().numpy()), bits(c))
    assert np.array_equal(bits(slot.scales.cpu().numpy()), bits(b))
    # the full-format reconstruction is close to the state
    err = (rt.reconstruct(slot) - dense).norm() / dense.norm()
    assert float(err) < 2e-2


def test_step_runs_the_decode_kernel_on_the_device(ssm_state):
    rt = runtime()
    bf = torch.bfloat16
    inputs = dict(query=torch.zeros((1, 1, HEADS // 2, 128), dtype=bf, device=DEV),
                  key=torch.zeros((1, 1, HEADS // 2, 128), dtype=bf, device=DEV),
                  value=torch.zeros((1, 1, HEADS, 128), dtype=bf, device=DEV),
                  log_decay=torch.zeros((1, 1, HEADS), device=DEV),
                  beta=torch.zeros((1, 1, HEADS), dtype=bf, device=DEV),
                  query_scale=128 ** -0.5)
    out = rt.step(ssm_state, 0, **inputs)
    torch.cuda.synchronize()
    assert out.shape == (1, 1, HEADS, 128) and out.dtype == bf
    # zero query and value: the output is exactly zero and one record is appended
    assert not out.float().any()
    slot = rt._slots[0]
    assert slot.steps == 1 and bool((slot.positions[:, 0] == 1).all())
    assert bool((slot.record_decay[:, 0] == 1.0).all())  # exp(0)
