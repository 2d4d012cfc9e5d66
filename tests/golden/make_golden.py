"""Generate the golden vectors in tests/golden from the reference library.

Run in the build container, where the reference's portable codec
(native/src of vLLM-HUST/gdn-state-codec) has been compiled from its own
sources into oracle/_ref/libgdn_ref.so by ``make -C oracle ref``:

    python tests/golden/make_golden.py

Everything written here comes out of the reference's public API
(GdnStateCodecCapsule::FromDenseBoundary -> Serialize / DenseState /
ApplyToken, and the Qwen layout adapter); see oracle/ref_shim.cpp.  Inputs
are seeded synthetic heads with the benchmark distribution (N(0,1) times a
per-head log-uniform factor in [1e-3, 1], 1% zeros) plus edge cases.  Queries
are rounded to bf16 values before they reach the reference, so the same
query feeds the bf16 CUDA entry points unchanged.

Files:
  reference_heads.npz  per head: dense input D [128,128] (capsule layout), the
                       serialized boundary (codes, smoothing, scales, rank-4
                       compensators K [128,4], V [128,4]), DenseState() and
                       the ApplyToken readout for query q.
  reference_small.npz  the same for the reference test's 8x6 state
                       (gdn_state_codec_state_capsule_test.cpp:40-48).
  adapter.npz          provider->capsule transpose of the reference adapter
                       test (gdn_state_codec_qwen38_gdn_adapter_test.cpp:20-31).
  reference_quant_only.npz
                       the reference's own quant-only stage (QuantizeBoundary,
                       DequantizeBoundary, ReadWindowState of capsule.cpp at
                       compensator rank 0, via oracle/ref_quant_shim.cpp) on
                       benchmark heads and edge cases: input, codes, smoothing,
                       scales, dense reconstruction, query and readout.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))

import oracle  # noqa: E402

OUT = Path(__file__).resolve().parent


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    bits = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16 << 16
    return rounded.astype(np.uint32).view(np.float32)


def benchmark_head(rng: np.random.Generator) -> np.ndarray:
    scale = 10.0 ** (-3.0 * rng.random())
    head = (rng.standard_normal((128, 128)) * scale).astype(np.float32)
    head[rng.random((128, 128)) < 0.01] = 0.0
    return head


def unit_query(rng: np.random.Generator, n: int = 128) -> np.ndarray:
    q = rng.standard_normal(n).astype(np.float32)
    q /= np.float32(np.linalg.norm(q))
    return bf16_round(q)


def main() -> None:
    if not oracle.ref_available():
        raise SystemExit("build the reference first: make -C oracle ref")
    rng = np.random.default_rng(0)
    heads = [benchmark_head(rng) for _ in range(3)]
    # Edge cases: one wide-range head (rows spanning 1e-6 .. 1e3) and one with
    # a zero row and a zero column.
    wide = (rng.standard_normal((128, 128)) *
            (10.0 ** rng.uniform(-6, 3, size=(128, 1)))).astype(np.float32)
    heads.append(wide)
    holes = benchmark_head(rng)
    holes[17, :] = 0.0
    holes[:, 90] = 0.0
    heads.append(holes)

    fields = {k: [] for k in ("dense", "query", "codes", "smoothing", "scales",
                              "compensator_keys", "compensator_values", "dense_state",
                              "projection")}
    for head in heads:
        q = unit_query(rng)
        result = oracle.ref_codec_head(head, q)
        fields["dense"].append(head)
        fields["query"].append(q)
        for key in ("codes", "smoothing", "scales", "compensator_keys",
                    "compensator_values", "dense_state", "projection"):
            fields[key].append(result[key])
    np.savez_compressed(OUT / "reference_heads.npz",
                        **{k: np.stack(v) for k, v in fields.items()})

    # The reference test's own 8x6 state (capsule_test.cpp:40-48).
    index = np.arange(48, dtype=np.float32)
    small = (np.sin((index + 1.0).astype(np.float32) * np.float32(0.37)).astype(np.float32)
             * np.float32(0.4)).astype(np.float32)
    small[np.arange(48) % 17 == 0] += np.float32(3.5)
    small = small.reshape(8, 6)
    qs = unit_query(rng, 8)
    r = oracle.ref_codec_head(small, qs)
    np.savez_compressed(OUT / "reference_small.npz", dense=small, query=qs,
                        **{k: r[k] for k in ("codes", "smoothing", "scales",
                                             "compensator_keys", "compensator_values",
                                             "dense_state", "projection")})

    provider = np.arange(1, 7, dtype=np.float32)  # [value=2][key=3]
    capsule = np.empty(6, np.float32)
    status = oracle.ref().ref_provider_to_capsule(
        provider.ctypes.data_as(oracle._f32p), 3, 2, capsule.ctypes.data_as(oracle._f32p))
    assert status == 0
    np.savez_compressed(OUT / "adapter.npz", provider=provider.reshape(2, 3),
                        capsule=capsule.reshape(3, 2))
    quant_only_fixture(rng)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


def quant_only_heads(rng: np.random.Generator) -> np.ndarray:
    """Two benchmark heads plus the edge cases the kernels special-case."""
    heads = [benchmark_head(rng), benchmark_head(rng)]
    heads.append(np.zeros((128, 128), np.float32))                       # all zero
    holes = benchmark_head(rng)
    holes[:, 3] = 0.0
    holes[9, :] = 0.0
    holes[50, 60] = -7.5                                                 # lone outlier
    heads.append(holes)
    heads.append((rng.standard_normal((128, 128)) * 1e-41).astype(np.float32))  # denormals
    wide = rng.standard_normal((128, 128)) * 10.0 ** rng.uniform(-30, 30, (128, 128))
    heads.append(wide.astype(np.float32))                                # wild range
    base = ((np.arange(128) % 127) + 0.5) * 2.0 ** -7                    # rounding ties
    base = base * (0.25 / base.mean())
    ties = np.stack([np.roll(base, k) for k in range(128)]).astype(np.float32)
    ties *= np.where(rng.random((128, 128)) < 0.5, -1, 1).astype(np.float32)
    heads.append(ties)
    heads.append((rng.integers(-127, 128, (128, 128)) * 2.0 ** -9).astype(np.float32))
    return np.stack(heads)


def quant_only_fixture(rng: np.random.Generator) -> None:
    if not oracle.ref_quant_available():
        raise SystemExit("build the reference first: make -C oracle ref")
    states = quant_only_heads(rng)
    codes, smoothing, scales = oracle.ref_quant_encode(states)
    dense = oracle.ref_quant_decode(codes, smoothing, scales)
    queries = np.stack([unit_query(rng) for _ in range(states.shape[0])])
    projection = oracle.ref_quant_project(codes, smoothing, scales, queries)
    np.savez_compressed(OUT / "reference_quant_only.npz", states=states, codes=codes,
                        smoothing=smoothing, scales=scales, dense=dense, query=queries,
                        projection=projection)


if __name__ == "__main__":
    main()
