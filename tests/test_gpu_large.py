"""GPU tests at sizes past 32-bit element offsets: one launch over 139,264
heads (2,281,701,376 elements > 2^31) for quantize, dequantize, the encoded
projection and the decode step, each checked bit for bit against the oracle
on heads near the start, the 2^31-element boundary and the end."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import codec

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
SLOTS, LAYERS, HEADS = 34, 32, 128   # 139,264 heads, 9.1 GB fp32
BOUNDARY_HEAD = 2**31 // (128 * 128)  # first head whose elements start at 2^31


def bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def large():
    free, _ = torch.cuda.mem_get_info(DEV)
    need = SLOTS * LAYERS * HEADS * (65536 * 2 + 17408 + 1024)
    if free < need + (4 << 30):
        pytest.skip(f"needs {need / 1e9:.1f} GB of device memory")
    states = codec.synthesize_states(SLOTS, LAYERS, HEADS, layout="provider", seed=17, device=DEV)
    states = states.reshape(-1, 128, 128)
    yield states
    del states
    torch.cuda.empty_cache()


def sample_heads(total: int) -> list[int]:
    return [0, 1, BOUNDARY_HEAD - 1, BOUNDARY_HEAD, BOUNDARY_HEAD + 1, total - 2, total - 1]


def test_quantize_dequantize_project_past_2g_elements(large):
    heads = large.shape[0]
    assert heads * 128 * 128 > 2**31
    enc = codec.quantize(large, "provider")
    dense = codec.dequantize(enc)
    queries = codec.synthesize_queries(1, 1, heads, seed=5, device=DEV).reshape(heads, 128)
    out = codec.encoded_projection(enc, queries)
    torch.cuda.synchronize()
    for h in sample_heads(heads):
        host = large[h:h + 1].cpu().numpy()
        z, c, b = oracle.quantize(host, "provider")
        assert np.array_equal(enc.codes[h:h + 1].cpu().numpy(), z), f"head {h} codes"
        assert np.array_equal(bits(enc.smoothing[h:h + 1].cpu().numpy()), bits(c)), f"head {h}"
        assert np.array_equal(bits(enc.scales[h:h + 1].cpu().numpy()), bits(b)), f"head {h}"
        assert np.array_equal(bits(dense[h:h + 1].cpu().numpy()),
                              bits(oracle.dequantize(z, c, b, layout="provider"))), f"head {h}"
        want = oracle.project(z, c, b, queries[h:h + 1].float().cpu().numpy(), layout="provider")
        assert np.array_equal(bits(out[h:h + 1].cpu().numpy()), bits(want)), f"head {h}"


def test_decode_step_past_2g_elements(large):
    heads = large.shape[0]
    window = codec.new_window(codec.quantize(large, "provider"))
    gen = torch.Generator(device=DEV).manual_seed(8)
    log_decay = -0.05 * torch.rand(heads, generator=gen, device=DEV)
    beta = torch.rand(heads, generator=gen, device=DEV).to(torch.bfloat16)
    kq = torch.randn((2, heads // 2, 128), generator=gen, device=DEV)
    kq = (kq / kq.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    values = torch.randn((heads, 128), generator=gen, device=DEV).to(torch.bfloat16)
    out = codec.window_step_bf16(window, log_decay, beta, kq[0], kq[1], values)
    torch.cuda.synchronize()
    bits16 = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    for h in sample_heads(heads):
        enc = window.encoded
        head = oracle.WindowHead(enc.codes[h].cpu().numpy(), enc.smoothing[h].cpu().numpy(),
                                 enc.scales[h].cpu().numpy(), layout="provider")
        alpha = float(window.record_decay[h, 0].cpu())
        token = oracle.qwen_token(alpha, bits16(beta[h:h + 1])[0], bits16(kq[0][h // 2]),
                                  bits16(kq[1][h // 2]), bits16(values[h]))
        want = head.step(*token, round_storage=True)
        assert np.array_equal(bits16(out[h]), oracle.f32_to_bf16_array(want)), f"head {h}"
        assert int(window.positions[h, 0].cpu()) == 1
