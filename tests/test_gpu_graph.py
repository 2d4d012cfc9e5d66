"""The codec's launches captured into a CUDA graph: quantize, dequantize, the
encoded projection and a decode step replayed from the graph give the same
bytes as the same calls made eagerly."""

from __future__ import annotations

import pytest
import torch

from gdn_state_codec import codec

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_graph_replay_matches_eager_launches():
    states = codec.synthesize_states(2, 2, 16, layout="provider", seed=81, device=DEV)
    queries = codec.synthesize_queries(2, 2, 16, seed=82, device=DEV)
    heads = states.numel() // (128 * 128)
    gen = torch.Generator(device=DEV).manual_seed(83)
    log_decay = -0.05 * torch.rand(heads, generator=gen, device=DEV)
    beta = torch.rand(heads, generator=gen, device=DEV).to(torch.bfloat16)
    kq = torch.randn((2, heads // 2, 128), generator=gen, device=DEV).to(torch.bfloat16)
    values = torch.randn((heads, 128), generator=gen, device=DEV).to(torch.bfloat16)

    def run(enc, dense, proj, window, out):
        codec.quantize(states, "provider", out=enc)
        codec.dequantize(enc, out=dense)
        codec.encoded_projection(enc, queries, out=proj)
        codec.window_step_bf16(window, log_decay, beta, kq[0], kq[1], values, out=out)

    def buffers():
        enc = codec.empty_encoded((2, 2, 16), "provider", DEV)
        dense = torch.empty_like(states)
        proj = torch.empty(queries.shape, dtype=torch.float32, device=DEV)
        window_enc = codec.quantize(states.reshape(heads, 128, 128), "provider")
        window = codec.new_window(window_enc)
        out = torch.empty((heads, 128), dtype=torch.bfloat16, device=DEV)
        return enc, dense, proj, window, out

    eager = buffers()
    run(*eager)  # also the first call on the device: set-up happens outside capture
    torch.cuda.synchronize()

    graphed = buffers()
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        run(*buffers())  # warm-up on the capture stream
    torch.cuda.current_stream(DEV).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    graphed[3].positions.zero_()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        run(*graphed)
    graph.replay()
    torch.cuda.synchronize()

    enc_e, dense_e, proj_e, window_e, out_e = eager
    enc_g, dense_g, proj_g, window_g, out_g = graphed
    assert torch.equal(enc_g.codes, enc_e.codes)
    assert torch.equal(enc_g.smoothing.view(torch.int32), enc_e.smoothing.view(torch.int32))
    assert torch.equal(enc_g.scales.view(torch.int32), enc_e.scales.view(torch.int32))
    assert torch.equal(dense_g.view(torch.int32), dense_e.view(torch.int32))
    assert torch.equal(proj_g.view(torch.int32), proj_e.view(torch.int32))
    assert torch.equal(out_g.view(torch.int16), out_e.view(torch.int16))
    assert torch.equal(window_g.record_keys.view(torch.int16), window_e.record_keys.view(torch.int16))
    assert bool((window_g.positions[:, 0] == 1).all())
