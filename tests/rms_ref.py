"""float32 restatement of the Llama RMSNorm + int8 quantiser's fixed
summation order, at TP=1 and split across tensor-parallel ranks.

The order is the definition that makes every tensor-parallel degree give the
same result (no counterpart in reef, whose GPT-Neo block uses LayerNorm, so
this restatement is the specification):

* a row of width W is 8 chunks of W/8 columns; a chunk is n4 = W/32 float4s;
* a chunk's sum of squares: 128 partials (partial i adds, in order, the
  float4s i, i + 128, ...; a float4 contributes ((a*a + b*b) + c*c) + d*d),
  an xor butterfly over each 32 partials, then ((w0 + w1) + w2) + w3;
* the row total is ((c0 + c1) + (c2 + c3)) + ((c4 + c5) + (c6 + c7));
* r = 1 / sqrt(total / W + eps), y = (x * gain) * r, scale =
  max|y| / 127 (1 for a zero row) with max|y| = max|x * gain| * r (rounding
  is monotonic), q = clamp(rint(y / scale), +-127).

A rank of an N-way group holds 8/N whole chunks, so it computes its chunk
sums and its max|x * gain| alone; the all-gathered (chunk sums, max) give
every rank TP=1's r and scale.
"""
import numpy as np

f32 = np.float32
CHUNKS = 8


def _butterfly(p):
    """xor-shuffle tree over the last axis (32 lanes, offsets 16..1)."""
    v = p.astype(f32, copy=True)
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        v = (v + v[..., lanes ^ o]).astype(f32)
    return v[..., 0]


def chunk_sums(x, width):
    """[rows][c * W/8] columns (whole chunks) -> [rows][c] chunk sums."""
    rows, cols = x.shape
    n4 = width // 32
    nch = cols // (4 * n4)
    a = x.reshape(rows, nch, n4, 4).astype(f32)
    sq = (((a[..., 0] * a[..., 0]).astype(f32) + (a[..., 1] * a[..., 1]).astype(f32)).astype(f32)
          + (a[..., 2] * a[..., 2]).astype(f32)).astype(f32)
    sq = (sq + (a[..., 3] * a[..., 3]).astype(f32)).astype(f32)
    steps = -(-n4 // 128)
    pad = np.zeros((rows, nch, steps * 128), f32)
    pad[..., :n4] = sq
    pad = pad.reshape(rows, nch, steps, 128)
    part = np.zeros((rows, nch, 128), f32)
    for k in range(steps):  # in order; adding a zero pad leaves a sum as it is
        part = (part + pad[:, :, k, :]).astype(f32)
    w = _butterfly(part.reshape(rows, nch, 4, 32))
    return (((w[..., 0] + w[..., 1]).astype(f32) + w[..., 2]).astype(f32) + w[..., 3]).astype(f32)


def finish(cs, gmax, width, eps):
    """From the 8 chunk sums [rows][8] and max|x * gain| [rows]: (r, scale)."""
    c = cs.astype(f32)
    t = ((((c[:, 0] + c[:, 1]).astype(f32) + (c[:, 2] + c[:, 3]).astype(f32)).astype(f32)
          + ((c[:, 4] + c[:, 5]).astype(f32) + (c[:, 6] + c[:, 7]).astype(f32)).astype(f32))
         .astype(f32))
    r = (f32(1) / np.sqrt((t / f32(width)).astype(f32) + f32(eps)).astype(f32)).astype(f32)
    mx = (gmax.astype(f32) * r).astype(f32)
    scale = np.where(mx > 0, (mx / f32(127)).astype(f32), f32(1)).astype(f32)
    return r, scale


def quantize(x, gain, r, scale):
    y = ((x * gain).astype(f32) * r[:, None]).astype(f32)
    return np.clip(np.rint((y / scale[:, None]).astype(f32)), -127, 127).astype(np.int8)


def rmsnorm_quant_ref(x, gain, eps):
    """TP=1: (q [rows][W] int8, scale [rows])."""
    width = x.shape[1]
    cs = chunk_sums(x, width)
    gmax = np.abs((x * gain).astype(f32)).max(axis=1)
    r, scale = finish(cs, gmax, width, eps)
    return quantize(x, gain, r, scale), scale


def rms_stats_local(x_local, gain_local, width):
    """A rank's pass 1 over its columns: [rows][chunks_local + 1] (its chunk
    sums, then its max|x * gain|)."""
    cs = chunk_sums(x_local, width)
    gmax = np.abs((x_local * gain_local).astype(f32)).max(axis=1)
    return np.concatenate([cs, gmax[:, None]], axis=1).astype(f32)


def rms_apply_local(x_local, gain_local, stats_all, width, eps):
    """A rank's pass 2 from the all-gathered stats [ranks][rows][chunks_local
    + 1]: (its q columns, scale)."""
    ranks, rows, s = stats_all.shape
    cs = np.concatenate([stats_all[g, :, :s - 1] for g in range(ranks)], axis=1)
    gmax = stats_all[:, :, s - 1].max(axis=0)
    r, scale = finish(cs, gmax, width, eps)
    return quantize(x_local, gain_local, r, scale), scale
