"""GPU parity of the slot-indexed entry points (ragged, non-contiguous int32
slot ids gathered / scattered by slot; config 4 of the benchmark plan at a
small size).  Indexing must be bit-exact: listed slots get exactly what the
dense kernels produce for them, every other slot is left untouched, padding
(-1) is skipped and invalid ids are reported, never trapped."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import codec

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
SLOTS, HPS = 48, 3  # cache of 48 slots x 3 heads


def sentinel_encoded(layout: str) -> codec.EncodedStates:
    enc = codec.empty_encoded((SLOTS, HPS), layout, DEV)
    enc.codes.fill_(0x55)
    enc.smoothing.fill_(-7.0)
    enc.scales.fill_(-9.0)
    return enc


@pytest.fixture(scope="module")
def cache():
    cap = codec.synthesize_states(SLOTS, 1, HPS, layout="capsule", seed=11, device=DEV)
    prov = codec.synthesize_states(SLOTS, 1, HPS, layout="provider", seed=11, device=DEV)
    return cap.reshape(SLOTS, HPS, 128, 128), prov.reshape(SLOTS, HPS, 128, 128)


def active_ids(count: int = 16, seed: int = 4) -> np.ndarray:
    return np.random.default_rng(seed).permutation(SLOTS)[:count].astype(np.int32)


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_quantize_indexed_scatter(cache, layout):
    states = cache[0] if layout == "capsule" else cache[1]
    ids = active_ids()
    enc = sentinel_encoded(layout)
    codec.quantize_indexed(states, enc, torch.from_numpy(ids).to(DEV), HPS)
    dense = codec.quantize(states[torch.from_numpy(ids).long().to(DEV)].contiguous(), layout)
    torch.cuda.synchronize()
    idx = torch.from_numpy(ids).long().to(DEV)
    assert torch.equal(enc.codes[idx], dense.codes)
    assert torch.equal(enc.smoothing[idx], dense.smoothing)
    assert torch.equal(enc.scales[idx], dense.scales)
    untouched = torch.ones(SLOTS, dtype=torch.bool, device=DEV)
    untouched[idx] = False
    assert bool((enc.codes[untouched] == 0x55).all())
    assert bool((enc.smoothing[untouched] == -7.0).all())
    # and against the oracle directly
    z, c, b = oracle.quantize(states[idx].reshape(-1, 128, 128).cpu().numpy(), layout)
    assert np.array_equal(enc.codes[idx].reshape(-1, 128, 128).cpu().numpy(), z)
    assert np.array_equal(enc.scales[idx].reshape(-1, 128).cpu().numpy().view(np.uint32),
                          b.view(np.uint32))


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_dequantize_and_projection_indexed(cache, layout):
    states = cache[0] if layout == "capsule" else cache[1]
    full = codec.quantize(states, layout)  # encode every slot
    ids = active_ids(seed=9)
    ids_pad = np.concatenate([ids[:5], [-1], ids[5:]]).astype(np.int32)  # PAD_SLOT_ID entry
    dev_ids = torch.from_numpy(ids_pad).to(DEV)
    out_cache = torch.full_like(states, 123.0)
    codec.dequantize_indexed(full, out_cache, dev_ids, HPS)
    q = codec.synthesize_queries(len(ids_pad), 1, HPS, seed=2, device=DEV).reshape(-1, HPS, 128)
    proj = codec.encoded_projection_indexed(full, q, dev_ids, HPS)
    dense_all = codec.dequantize(full)
    torch.cuda.synchronize()
    idx = torch.from_numpy(ids).long().to(DEV)
    assert torch.equal(out_cache[idx], dense_all[idx])
    mask = torch.ones(SLOTS, dtype=torch.bool, device=DEV)
    mask[idx] = False
    assert bool((out_cache[mask] == 123.0).all())
    # projection rows follow the batch order; the padded entry outputs zeros
    assert bool((proj[5] == 0).all())
    gather = torch.from_numpy(np.concatenate([ids[:5], ids[5:]])).long().to(DEV)
    q_real = torch.cat([q[:5], q[6:]])
    sub = codec.EncodedStates(full.codes[gather].contiguous(), full.smoothing[gather].contiguous(),
                              full.scales[gather].contiguous(), layout)
    dense_proj = codec.encoded_projection(sub, q_real.contiguous())
    assert torch.equal(torch.cat([proj[:5], proj[6:]]), dense_proj)


def test_invalid_slot_ids_are_reported_not_trapped(cache):
    states = cache[0]
    codec.device_error(DEV, clear=True)
    ids = torch.tensor([3, SLOTS, -1, 7, -5], dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    enc = sentinel_encoded("capsule")
    codec.quantize_indexed(states, enc, ids, HPS, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1 == 1
    assert codec.device_error(DEV, clear=True) & 1 == 1
    assert codec.device_error(DEV) == 0
    ok = torch.tensor([3, 7], dtype=torch.long, device=DEV)
    dense = codec.quantize(states[ok].contiguous(), "capsule")
    assert torch.equal(enc.codes[ok], dense.codes)
    bad_free = torch.ones(SLOTS, dtype=torch.bool, device=DEV)
    bad_free[ok] = False
    assert bool((enc.codes[bad_free] == 0x55).all())
    # The context is still usable after the report.
    again = codec.quantize(states[3:4].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(again.codes, enc.codes[3:4])
