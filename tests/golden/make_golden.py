"""Writes the golden fixtures under tests/golden (run in a container with gguf-py).

  q8_0_gguf.npz   f16 input groups and their Q8_0 encoding by gguf-py 0.19's
                  numpy Q8_0 (``gguf.quants.quantize(x, Q8_0)``), the
                  implementation that gguf-py documents as bit-exact with
                  GGML's reference quantizer.  Inputs: seeded N(0,1) rows,
                  rows with 8-sigma outliers, all-zero groups, tiny groups
                  whose scale is an f16 subnormal, groups at the f16 maximum,
                  and groups built so that x/d lands on .5 ties.
  probe_pages.npz the decode probe's page order: xorshift32 Fisher-Yates with
                  seed 0x9e3779b9 (src/bin/decode_gqa_probe.rs:13-23), for the
                  probe's pool of ceil(1025/64)+7 = 24 pages and for 257 pages,
                  computed here by a pure-Python restatement that is
                  independent of the oracle's C code.

Usage: python tests/golden/make_golden.py
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def q8_inputs() -> np.ndarray:
    rng = np.random.default_rng(20260824)
    rows = [rng.standard_normal((64, 32))]
    out = rng.standard_normal((64, 32))
    mask = rng.random((64, 32)) < 0.05
    out[mask] = 8.0 * np.sign(rng.standard_normal(mask.sum()))
    rows.append(out)
    rows.append(np.zeros((4, 32)))
    rows.append(rng.standard_normal((8, 32)) * 1e-4)       # subnormal f16 scales
    rows.append(rng.standard_normal((8, 32)) * 1e-6)       # inputs themselves subnormal
    big = rng.standard_normal((4, 32)) * 1e4
    big[:, 0] = 65504.0
    rows.append(big)
    ties = np.tile(np.arange(-16, 16, dtype=np.float64) + 0.5, (4, 1))
    ties[:, -1] = 127.0                                     # amax 127 -> d = 1, x*id = k+0.5
    rows.append(ties)
    ties2 = np.tile(np.linspace(-63.5, 63.5, 32), (4, 1))
    ties2[:, 0] = -127.0
    rows.append(ties2)
    x = np.concatenate(rows, axis=0).astype(np.float16)
    return x


def xorshift_pages(count: int, seed: int = 0x9E3779B9) -> np.ndarray:
    pages = list(range(count))
    state = seed
    for i in range(count - 1, 0, -1):
        state ^= (state << 13) & 0xFFFFFFFF
        state ^= state >> 17
        state ^= (state << 5) & 0xFFFFFFFF
        j = state % (i + 1)
        pages[i], pages[j] = pages[j], pages[i]
    return np.asarray(pages, np.uint32)


def main() -> None:
    import gguf
    from gguf.quants import quantize

    x = q8_inputs()
    enc = quantize(x.astype(np.float32), gguf.GGMLQuantizationType.Q8_0)  # [rows, 34] bytes per group
    enc = np.asarray(enc, np.uint8).reshape(x.shape[0], 34)
    d = enc[:, :2].copy().view(np.float16).reshape(-1)
    qs = enc[:, 2:].copy().view(np.int8)
    np.savez_compressed(os.path.join(HERE, "q8_0_gguf.npz"), x=x, d=d, qs=qs,
                        gguf_version=np.asarray(getattr(gguf, "__version__", "0.19.0")))
    np.savez_compressed(os.path.join(HERE, "probe_pages.npz"), pages24=xorshift_pages(24),
                        pages257=xorshift_pages(257))
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
