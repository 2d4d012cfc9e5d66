"""Slot-indexed parity at the ragged benchmark configuration's exact geometry.

A 1,024-slot x 30-layer x 32-head cache (983,040 heads: 64 GB of fp32 state
and 17 GB encoded), of which 256 slots, the first 256 of a seeded permutation
of 0..1023 (int32, non-contiguous, the same ids bench.py times), are
quantized, projected and dequantized back into the cache by slot id.  For
each layout:

* every active slot's codes, smoothing and scales equal the dense kernel's
  result on the gathered slots, and every projection output and dequantized
  head equals the dense kernels' on the gathered encodings (device against
  device, bit for bit);
* every inactive slot is untouched: its encoded planes still hold a sentinel,
  and its fp32 state keeps its checksum through the scatter of the
  dequantize;
* a seeded sample of 512 heads spread over the active slots, layers and heads
  is bit-exact to the CPU oracle (oracle.quantize / project / dequantize),
  the restatement of native/src/gdn_state_codec_state_capsule.cpp:190-304
  pinned to the reference library.

The reference's own check of a whole device batch against its host oracle
is native/ascendc/gdn_state_codec/host/gdn_state_codec_provider_quantize_
probe.cpp:127-183.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import codec

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
CACHE_SLOTS, ACTIVE, LAYERS, HEADS = 1024, 256, 30, 32
PER_SLOT = LAYERS * HEADS
SAMPLE = 512
CHUNK = 16  # slots per device-against-device comparison
SENTINEL_CODE, SENTINEL_FLOAT = 90, -7.0


def bits(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int32) if t.dtype == torch.float32 else t


def same(a: torch.Tensor, b: torch.Tensor) -> bool:
    return torch.equal(bits(a), bits(b))


def slot_checksums(states: torch.Tensor) -> torch.Tensor:
    """Per-slot int64 sum of the fp32 bit patterns, a few slots at a time."""
    words = states.view(torch.int32).view(CACHE_SLOTS, -1)
    return torch.cat([words[i:i + CHUNK].sum(dim=1, dtype=torch.int64)
                      for i in range(0, CACHE_SLOTS, CHUNK)])


def gathered(encoded: codec.EncodedStates, ids: torch.Tensor) -> codec.EncodedStates:
    return codec.EncodedStates(encoded.codes.index_select(0, ids),
                               encoded.smoothing.index_select(0, ids),
                               encoded.scales.index_select(0, ids), encoded.layout)


@pytest.fixture(scope="module", autouse=True)
def enough_memory():
    need = CACHE_SLOTS * PER_SLOT * (65536 + 16384 + 1024) + (8 << 30)
    free, _ = torch.cuda.mem_get_info(DEV)
    if free < need:
        pytest.skip(f"config-4 geometry needs {need / 1e9:.0f} GB, {free / 1e9:.0f} GB free")


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_config4_geometry(layout):
    states = codec.synthesize_states(CACHE_SLOTS, LAYERS, HEADS, layout=layout, seed=5,
                                     device=DEV)
    cache = codec.empty_encoded((CACHE_SLOTS, LAYERS, HEADS), layout, DEV)
    cache.codes.fill_(SENTINEL_CODE)
    cache.smoothing.fill_(SENTINEL_FLOAT)
    cache.scales.fill_(SENTINEL_FLOAT)
    perm = torch.randperm(CACHE_SLOTS, generator=torch.Generator().manual_seed(0))
    ids_cpu = perm[:ACTIVE].to(torch.int32)
    ids = ids_cpu.to(DEV)
    ids_long = ids.long()
    inactive = torch.ones(CACHE_SLOTS, dtype=torch.bool)
    inactive[perm[:ACTIVE]] = False
    inactive_ids = inactive.nonzero().flatten().to(DEV)
    queries = codec.synthesize_queries(ACTIVE, LAYERS, HEADS, seed=9, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    checksums = slot_checksums(states)

    # -- quantize by slot id ----------------------------------------------------
    codec.quantize_indexed(states, cache, ids, PER_SLOT, status=status)
    outputs = codec.encoded_projection_indexed(cache, queries, ids, PER_SLOT, status=status)
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0
    for c0 in range(0, ACTIVE, CHUNK):
        chunk = ids_long[c0:c0 + CHUNK]
        dense_enc = codec.quantize(states.index_select(0, chunk), layout)
        got = gathered(cache, chunk)
        assert same(got.codes, dense_enc.codes), f"codes of slots {chunk.tolist()}"
        assert same(got.smoothing, dense_enc.smoothing)
        assert same(got.scales, dense_enc.scales)
        want = codec.encoded_projection(dense_enc, queries[c0:c0 + CHUNK])
        assert same(outputs[c0:c0 + CHUNK], want)
    for c0 in range(0, inactive_ids.numel(), 4 * CHUNK):
        chunk = inactive_ids[c0:c0 + 4 * CHUNK]
        assert bool((cache.codes.index_select(0, chunk) == SENTINEL_CODE).all())
        assert bool((cache.smoothing.index_select(0, chunk) == SENTINEL_FLOAT).all())
        assert bool((cache.scales.index_select(0, chunk) == SENTINEL_FLOAT).all())

    # -- the oracle on a seeded sample of heads -----------------------------------
    rng = np.random.default_rng(17)
    entries = rng.integers(0, ACTIVE, SAMPLE)
    within = rng.integers(0, PER_SLOT, SAMPLE)  # layer * 32 + head
    flat = torch.as_tensor(ids_cpu.numpy().astype(np.int64)[entries] * PER_SLOT + within,
                           device=DEV)
    def sample(t):
        return t.reshape(CACHE_SLOTS * PER_SLOT, *t.shape[3:]).index_select(0, flat).cpu().numpy()
    host_states = sample(states)
    z, c, b = sample(cache.codes), sample(cache.smoothing), sample(cache.scales)
    wz, wc, wb = oracle.quantize(host_states, layout, threads=8)
    assert np.array_equal(z, wz)
    assert np.array_equal(c.view(np.uint32), wc.view(np.uint32))
    assert np.array_equal(b.view(np.uint32), wb.view(np.uint32))
    q = queries.reshape(ACTIVE * PER_SLOT, 128)[torch.as_tensor(entries * PER_SLOT + within,
                                                                device=DEV)]
    o = outputs.reshape(ACTIVE * PER_SLOT, 128)[torch.as_tensor(entries * PER_SLOT + within,
                                                                device=DEV)]
    want_o = oracle.project(wz, wc, wb, q.float().cpu().numpy(), layout=layout)
    assert np.array_equal(o.cpu().numpy().view(np.uint32), want_o.view(np.uint32))

    # -- dequantize by slot id back into the fp32 cache ------------------------------
    codec.dequantize_indexed(cache, states, ids, PER_SLOT, status=status)
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0
    for c0 in range(0, ACTIVE, CHUNK):
        chunk = ids_long[c0:c0 + CHUNK]
        want = codec.dequantize(gathered(cache, chunk))
        assert same(states.index_select(0, chunk), want)
    after = slot_checksums(states)
    assert torch.equal(after[inactive_ids], checksums[inactive_ids])
    want_d = oracle.dequantize(wz, wc, wb, layout=layout, threads=8)
    assert np.array_equal(sample(states).view(np.uint32), want_d.view(np.uint32))
    del states, cache, queries, outputs
    torch.cuda.empty_cache()
