"""Packed weight / activation formats and their quantizers (load time, numpy).

The packed layouts are lowbit's, byte for byte (src/lowbit/csrc/lowbit.h:9-19,
src/lowbit/formats.py), so weights packed by lowbit load unchanged and the
quantizers below produce bit-identical packed arrays for the same inputs:

* int4, group 128: ``qw`` uint8 [N, Kp/2]; within group g (bytes 64g..64g+63)
  byte j holds element 128g+j (low nibble) and 128g+64+j (high nibble);
  value = (q - z) * s, z = 8 when ``zeros`` is None.
* MXFP4, block 32: ``qw`` uint8 [N, Kp/2]; within block b (bytes 16b..16b+15)
  byte j holds element 32b+j (low) and 32b+16+j (high) as OCP E2M1 codes;
  value = e2m1(q) * 2^(e8m0 - 127), e8m0 = 255 is NaN.
* int8 activations: per-token scale absmax/127, codes clipped to +-127, and
  per-group (128) code sums.

Quantization runs once at load time on the host (as in the reference); the
GPU consumes the packed arrays. Containers hold numpy arrays or torch tensors;
``.cuda()`` returns a copy whose arrays are torch CUDA tensors.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

GROUP = 128
MXBLOCK = 32

# OCP E2M1 code -> value: bit 3 sign, bits 2..1 exponent (bias 1), bit 0 mantissa
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)
E2M1_EMAX = 2  # exponent of 6.0 = 1.5 * 2^2, the largest E2M1 magnitude


def pad_to(k: int, block: int) -> int:
    """Smallest multiple of ``block`` that is >= k."""
    return ((k + block - 1) // block) * block


def _np(a):
    """numpy view of a numpy array or a (possibly CUDA) torch tensor."""
    if isinstance(a, np.ndarray) or a is None:
        return a
    return a.detach().cpu().numpy()


def _nbytes(a) -> int:
    if a is None:
        return 0
    if hasattr(a, "element_size"):  # torch tensor
        return int(a.numel()) * int(a.element_size())
    return int(a.nbytes)


# ---------------------------------------------------------------- nibble packing

def pack_nibbles(codes: np.ndarray, block: int) -> np.ndarray:
    """Pack 4-bit codes [N, Kp] into bytes [N, Kp/2], per block: byte j = code j | code j+block/2 << 4."""
    codes = np.asarray(codes)
    n, kp = codes.shape
    if kp % block:
        raise ValueError(f"Kp={kp} is not a multiple of the block size {block}")
    half = block // 2
    c = codes.astype(np.uint8).reshape(n, kp // block, block)
    return (c[:, :, :half] | (c[:, :, half:] << 4)).reshape(n, kp // 2)


def unpack_nibbles(packed: np.ndarray, block: int) -> np.ndarray:
    """Inverse of pack_nibbles."""
    packed = _np(packed)
    n, nbytes = packed.shape
    p = packed.reshape(n, (2 * nbytes) // block, block // 2)
    return np.concatenate([p & 15, p >> 4], axis=2).reshape(n, 2 * nbytes)


# ---------------------------------------------------------------- containers

@dataclass
class Int4Weights:
    """int4 weights, group 128, fp32 scale per group, optional uint8 zero-point."""
    qw: object            # uint8 [N, Kp/2]
    scales: object        # float32 [N, G]
    zeros: object | None  # uint8 [N, G] or None (symmetric, z = 8)
    k: int                # logical K before padding

    @property
    def n(self) -> int:
        return int(self.qw.shape[0])

    @property
    def kp(self) -> int:
        return int(self.qw.shape[1]) * 2

    @property
    def nbytes(self) -> int:
        return _nbytes(self.qw) + _nbytes(self.scales) + _nbytes(self.zeros)

    def codes(self) -> np.ndarray:
        return unpack_nibbles(self.qw, GROUP)

    def dequantize(self) -> np.ndarray:
        """[N, K] float32 (references and tests only; the kernels never expand W)."""
        q = self.codes().astype(np.float32).reshape(self.n, -1, GROUP)
        z = np.float32(8) if self.zeros is None else _np(self.zeros).astype(np.float32)[:, :, None]
        w = (q - z) * _np(self.scales)[:, :, None]
        return w.reshape(self.n, self.kp)[:, : self.k]

    def cuda(self, device=None) -> "Int4Weights":
        from ._torch import to_cuda
        return replace(self, qw=to_cuda(self.qw, device), scales=to_cuda(self.scales, device),
                       zeros=None if self.zeros is None else to_cuda(self.zeros, device))

    def shard(self, rank: int, world: int) -> "Int4Weights":
        """Rows [rank*N/world, (rank+1)*N/world) (column-parallel N-sharding)."""
        lo, hi = shard_bounds(self.n, rank, world)
        return replace(self, qw=self.qw[lo:hi], scales=self.scales[lo:hi],
                       zeros=None if self.zeros is None else self.zeros[lo:hi])


@dataclass
class MXFP4Weights:
    """OCP MXFP4: E2M1 elements in blocks of 32 sharing an E8M0 scale 2^(e - 127)."""
    qw: object    # uint8 [N, Kp/2]
    e8m0: object  # uint8 [N, Kp/32]
    k: int

    @property
    def n(self) -> int:
        return int(self.qw.shape[0])

    @property
    def kp(self) -> int:
        return int(self.qw.shape[1]) * 2

    @property
    def nbytes(self) -> int:
        return _nbytes(self.qw) + _nbytes(self.e8m0)

    def codes(self) -> np.ndarray:
        return unpack_nibbles(self.qw, MXBLOCK)

    def dequantize(self) -> np.ndarray:
        v = E2M1_VALUES[self.codes()].reshape(self.n, -1, MXBLOCK)
        return (v * e8m0_to_float(_np(self.e8m0))[:, :, None]).reshape(self.n, self.kp)[:, : self.k]

    def cuda(self, device=None) -> "MXFP4Weights":
        from ._torch import to_cuda
        return replace(self, qw=to_cuda(self.qw, device), e8m0=to_cuda(self.e8m0, device))

    def shard(self, rank: int, world: int) -> "MXFP4Weights":
        lo, hi = shard_bounds(self.n, rank, world)
        return replace(self, qw=self.qw[lo:hi], e8m0=self.e8m0[lo:hi])


@dataclass
class Int8Acts:
    """Per-token int8 activations with per-group code sums."""
    xq: object     # int8 [M, Kp]
    scale: object  # float32 [M]
    gsum: object   # int32 [M, Kp/128]

    def dequantize(self) -> np.ndarray:
        return _np(self.xq).astype(np.float32) * _np(self.scale)[:, None]


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous row range of `rank` when n rows are split over `world` ranks
    (the first n % world ranks get one extra row)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


# ---------------------------------------------------------------- int4 quantizer

def quantize_int4(w: np.ndarray, asym: bool = False, scale: str = "absmax") -> Int4Weights:
    """Round-to-nearest int4, group 128 along K (lowbit's rule, src/lowbit/formats.py:90-142).

    absmax (default): s = max|w|/7, q = clip(rint(w/s), -8, 7) + 8
    signed-max      : s = m/-8 with m the group's largest-magnitude element
                      (sign kept; 16 levels used, s may be negative), same q
    asym            : s = (max(w,0) - min(w,0))/15, z = clip(rint(-min/s), 0, 15),
                      q = clip(rint(w/s) + z, 0, 15)
    A zero scale becomes 1. Padded elements get the code that decodes to 0.
    """
    if scale not in ("absmax", "signed-max"):
        raise ValueError(f"scale must be 'absmax' or 'signed-max', not {scale!r}")
    if asym and scale != "absmax":
        raise ValueError("scale='signed-max' is a symmetric rule (asym=False)")
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    kp = pad_to(k, GROUP)
    ng = kp // GROUP
    wpad = np.zeros((n, kp), np.float32)
    wpad[:, :k] = w
    grp = wpad.reshape(n, ng, GROUP)
    live = (np.arange(kp) < k).reshape(1, ng, GROUP)
    one = np.float32(1.0)
    if asym:
        hi = np.maximum(np.where(live, grp, -np.inf).max(axis=2), 0.0).astype(np.float32)
        lo = np.minimum(np.where(live, grp, np.inf).min(axis=2), 0.0).astype(np.float32)
        s = ((hi - lo) / np.float32(15)).astype(np.float32)
        s = np.where(s > 0, s, one).astype(np.float32)
        z = np.clip(np.rint(-lo / s), 0, 15).astype(np.uint8)
        q = np.clip(np.rint(grp / s[..., None]) + z[..., None], 0, 15)
        q = np.where(live, q, z[..., None])
        zeros = z
    else:
        if scale == "signed-max":
            pick = np.abs(grp).argmax(axis=2)[..., None]
            s = (np.take_along_axis(grp, pick, axis=2)[..., 0] / np.float32(-8)).astype(np.float32)
            s = np.where(s != 0, s, one).astype(np.float32)
        else:
            s = (np.abs(grp).max(axis=2) / np.float32(7)).astype(np.float32)
            s = np.where(s > 0, s, one).astype(np.float32)
        q = np.clip(np.rint(grp / s[..., None]), -8, 7) + 8
        q = np.where(live, q, 8)
        zeros = None
    codes = q.astype(np.uint8).reshape(n, kp)
    return Int4Weights(pack_nibbles(codes, GROUP), s.astype(np.float32), zeros, k)


# ---------------------------------------------------------------- MXFP4 quantizer

def e8m0_to_float(e: np.ndarray) -> np.ndarray:
    """E8M0 biased exponent -> 2^(e-127) as float32; 255 -> NaN, 0 -> 2^-127."""
    e = np.asarray(e, dtype=np.uint8)
    out = np.ldexp(np.float32(1.0), np.where(e == 255, 0, e.astype(np.int32) - 127)).astype(np.float32)
    return np.where(e == 255, np.float32(np.nan), out).astype(np.float32)


def fp32_to_e2m1(v: np.ndarray) -> np.ndarray:
    """Round (already block-scaled) fp32 values to E2M1 codes: nearest, ties to
    the even mantissa, saturating at +-6; -0 and values rounding to 0 get code 0."""
    v = np.asarray(v, np.float32)
    a = np.abs(v)
    # decision points between the magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6; a tie
    # (.25, .75, 1.25, 1.75, 2.5, 3.5, 5) goes to the neighbour with an even code
    mag = np.zeros(a.shape, np.uint8)
    for cut, inclusive in ((0.25, False), (0.75, True), (1.25, False), (1.75, True),
                           (2.5, False), (3.5, True), (5.0, False)):
        mag += (a >= cut) if inclusive else (a > cut)
    neg = (np.signbit(v) & (mag > 0)).astype(np.uint8)
    return (mag | (neg << 3)).astype(np.uint8)


def quantize_mxfp4(w: np.ndarray) -> MXFP4Weights:
    """OCP MX v1.0: per block of 32, shared exponent floor(log2(amax)) - 2 (src/lowbit/formats.py:197-212)."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    kp = pad_to(k, MXBLOCK)
    wpad = np.zeros((n, kp), np.float32)
    wpad[:, :k] = w
    blk = wpad.reshape(n, kp // MXBLOCK, MXBLOCK)
    amax = np.abs(blk).max(axis=2)
    nz = amax > 0
    lg = np.zeros_like(amax)
    np.log2(amax, where=nz, out=lg)
    shared = np.where(nz, np.floor(lg) - E2M1_EMAX, 0)
    e = np.clip(shared + 127, 0, 254).astype(np.uint8)
    codes = fp32_to_e2m1(blk / e8m0_to_float(e)[..., None]).reshape(n, kp)
    return MXFP4Weights(pack_nibbles(codes, MXBLOCK), e, k)


# ---------------------------------------------------------------- activations

def pad_acts(x: np.ndarray, kp: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.shape[1] == kp:
        return x
    out = np.zeros((x.shape[0], kp), np.float32)
    out[:, : x.shape[1]] = x
    return out


def quantize_act_int8(x: np.ndarray, kp: int | None = None) -> Int8Acts:
    """Per-token symmetric int8 (numpy): s = absmax/127 (1 for a zero row),
    q = clip(rint(x/s), -127, 127); bit-identical to the GPU quantizer."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    kp = pad_to(x.shape[1], GROUP) if kp is None else kp
    xp = pad_acts(x, kp)
    amax = np.abs(xp).max(axis=1)
    s = np.where(amax > 0, amax / np.float32(127), np.float32(1)).astype(np.float32)
    q = np.clip(np.rint(xp / s[:, None]), -127, 127).astype(np.int8)
    gsum = q.reshape(q.shape[0], -1, GROUP).astype(np.int32).sum(axis=2, dtype=np.int32)
    return Int8Acts(q, s, gsum)


# ---------------------------------------------------------------- AMX repack (drop-in)

@dataclass
class AMXInt4Weights:
    """int4 g128 weights in the layout of lowbit's AMX tile kernel
    (src/lowbit/formats.py:251-293), kept byte for byte so that weights a
    lowbit caller repacked with its `pack_amx` are accepted unchanged.

    Per block of 16 output rows and group g: 1 KiB where byte (r, 4c + i) holds
    the code of row n0 + c at element 128g + 4r + i (low nibble) and at
    128g + 64 + 4r + i (high nibble); scales s, s * z and z as [NB, G, 16].
    On the GPU these weights run the W4A8 kernels in the canonical layout:
    `to_int4()` undoes the repack exactly (padding rows dropped)."""
    qw: np.ndarray      # uint8 [NB * G * 1024]
    scales: np.ndarray  # float32 [NB, G, 16]
    sz: np.ndarray      # float32 [NB, G, 16]  = s * z
    zeros: np.ndarray   # uint8 [NB, G, 16]
    n: int
    k: int
    kp: int

    @property
    def nbytes(self) -> int:
        return self.qw.nbytes + self.scales.nbytes + self.sz.nbytes

    def to_int4(self) -> Int4Weights:
        """The canonical Int4Weights these bytes were packed from: byte (r, c, i)
        of block b, group g is byte j = 4r + i of row 16b + c's group g (the
        canonical layout puts element 128g + j in the low nibble of that byte and
        128g + 64 + j in the high one, as the AMX layout does)."""
        nb, g = self.scales.shape[0], self.kp // GROUP
        b = np.asarray(self.qw, np.uint8).reshape(nb, g, 16, 16, 4)          # [nb, g, r, c, i]
        qw = np.ascontiguousarray(b.transpose(0, 3, 1, 2, 4)).reshape(nb * 16, g * 64)[: self.n]
        sc = np.ascontiguousarray(np.asarray(self.scales, np.float32).transpose(0, 2, 1)).reshape(nb * 16, g)
        z = np.ascontiguousarray(np.asarray(self.zeros, np.uint8).transpose(0, 2, 1)).reshape(nb * 16, g)
        return Int4Weights(qw, sc[: self.n].copy(), z[: self.n].copy(), self.k)


def pack_amx(w: Int4Weights) -> AMXInt4Weights:
    """The AMX repack of lowbit (src/lowbit/formats.py:275-293): rows padded to
    a multiple of 16 with codes equal to their zero point (they decode to 0)."""
    n, kp = w.n, w.kp
    g = kp // GROUP
    nb = -(-n // 16)
    z = np.full((nb * 16, g), 8, np.uint8)
    if w.zeros is not None:
        z[:n] = _np(w.zeros)
    s = np.zeros((nb * 16, g), np.float32)
    s[:n] = _np(w.scales)
    # canonical bytes of padding rows: both nibbles = z
    qw = np.empty((nb * 16, kp // 2), np.uint8)
    qw[:n] = _np(w.qw)
    qw[n:] = np.repeat(z[n:] * np.uint8(17), 64, axis=1)
    # [nb, c, g, r, i] -> [nb, g, r, c, i]
    packed = qw.reshape(nb, 16, g, 16, 4).transpose(0, 2, 3, 1, 4)
    sb = np.ascontiguousarray(s.reshape(nb, 16, g).transpose(0, 2, 1))
    zb = np.ascontiguousarray(z.reshape(nb, 16, g).transpose(0, 2, 1))
    return AMXInt4Weights(np.ascontiguousarray(packed).reshape(-1), sb,
                          (sb * zb.astype(np.float32)).astype(np.float32), zb, n, w.k, kp)

