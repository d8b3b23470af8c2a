"""Generate the golden fixtures in tests/golden/ (run from the repo root:
``python tests/golden/make_golden.py``).

The reference (lmrs) ships no tests or vectors for the quantized path, so the
fixtures come from sources independent of the oracle under test:

* ``awq_kat.npz``   — AWQ known-answer vectors written from the format text
  (nibble i of word j = column 8j + ORDER[i], ORDER = [0,2,4,6,1,3,5,7]) with
  explicit per-nibble Python loops, plus a small dequant/linear case whose
  expected weights are float64 products rounded once to fp16.
* ``e4m3.npz``      — torch's ``float8_e4m3fn`` cast (an independent encoder) on
  a value sweep, and the decoded value of every byte.
* ``fp8_quant.npz`` — per-row quantisation (s = absmax/448 in fp32, q = e4m3(x/s))
  computed with torch on CPU.

Every random draw is seeded; rerunning reproduces the files bit for bit.
"""
import pathlib

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
ORDER = [0, 2, 4, 6, 1, 3, 5, 7]


def pack_loops(q):
    R, C = q.shape
    out = np.zeros((R, C // 8), dtype=np.uint32)
    for r in range(R):
        for j in range(C // 8):
            w = 0
            for i in range(8):
                w |= (int(q[r, 8 * j + ORDER[i]]) & 0xF) << (4 * i)
            out[r, j] = w
    return out.view(np.int32)


def unpack_loops(words):
    words = np.asarray(words).view(np.uint32)
    R, W = words.shape
    out = np.zeros((R, W * 8), dtype=np.int8)
    for r in range(R):
        for j in range(W):
            w = int(words[r, j])
            for i in range(8):
                out[r, 8 * j + ORDER[i]] = (w >> (4 * i)) & 0xF
    return out


def awq_kat():
    words = np.array([[0x00000000, 0xFFFFFFFF, 0x76543210, 0x01234567],
                      [0x80000001, 0x0F0F0F0F, 0x12345678, 0xDEADBEEF]], dtype=np.uint32)
    unpacked = unpack_loops(words)
    # hand check of one word: 0x76543210 has nibble i == i, so column ORDER[i] == i
    assert list(unpacked[0, 16:24]) == [0, 4, 1, 5, 2, 6, 3, 7]
    rng = np.random.default_rng(1234)
    K, N, g, M = 256, 64, 128, 4
    q = rng.integers(0, 16, size=(K, N)).astype(np.int8)
    z = rng.integers(0, 16, size=(K // g, N)).astype(np.int8)
    s = rng.uniform(0.001, 0.02, size=(K // g, N)).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    qw, qz = pack_loops(q), pack_loops(z)
    w = np.empty((K, N), np.float16)
    for k in range(K):
        gi = k // g
        w[k] = ((q[k].astype(np.float64) - z[gi].astype(np.float64)) * s[gi].astype(np.float64)).astype(np.float16)
    y64 = x.astype(np.float64) @ w.astype(np.float64)
    np.savez_compressed(HERE / "awq_kat.npz", words=words.view(np.int32), unpacked=unpacked,
             q=q, z=z, qweight=qw, qzeros=qz, scales=s, x=x, w=w, y64=y64, group=g)


def e4m3():
    vals = np.concatenate([
        np.linspace(-470.0, 470.0, 18801, dtype=np.float32),
        np.ldexp(np.float32(1.0), np.arange(-12, 9)).astype(np.float32),
        -np.ldexp(np.float32(1.0), np.arange(-12, 9)).astype(np.float32),
        (np.random.default_rng(7).standard_normal(20000) * 20).astype(np.float32),
        np.array([0.0, -0.0, 448.0, -448.0, 463.9, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11],
                 dtype=np.float32),
    ])
    # torch's cast does not saturate: whatever rounds up to 480 becomes NaN, while
    # cvt.rn.satfinite gives 448.  Below 464 (the 448/480 midpoint) the two agree.
    vals = vals[np.abs(vals) < 464.0]
    enc = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    codes = np.arange(256, dtype=np.uint8)
    dec = torch.from_numpy(codes).view(torch.float8_e4m3fn).to(torch.float32).numpy()
    np.savez_compressed(HERE / "e4m3.npz", values=vals, codes=enc, decoded=dec)


def fp8_quant():
    rng = np.random.default_rng(99)
    x = torch.from_numpy((rng.standard_normal((6, 256)) *
                          rng.uniform(0.01, 50.0, size=(6, 1))).astype(np.float32)).bfloat16()
    x[0] = 0
    x[1, 17] = 3000.0
    xf = x.float()
    s = xf.abs().amax(dim=1) / 448.0
    q = torch.where(s[:, None] == 0, torch.zeros_like(xf), xf / s[:, None])
    qb = q.to(torch.float8_e4m3fn).view(torch.uint8)
    qb[s == 0] = 0
    np.savez_compressed(HERE / "fp8_quant.npz", x_bf16=x.view(torch.int16).numpy().view(np.uint16),
             q=qb.numpy(), s=s.numpy())


if __name__ == "__main__":
    awq_kat()
    e4m3()
    fp8_quant()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
