"""Codecs and scalar rules of the monokernel path, restated on the CPU (oracle; tests only).

Every function here is element-wise and bit-exact: the CUDA kernels must produce
the same bits for the same inputs. Citations are to omirosh/sgl-amd-mono.
"""

from __future__ import annotations

import math

import numpy as np
import torch

FP8_MAX = 448.0
FLT_MIN = 1.1754943508222875e-38
# E2M1 values by code (bit 3 = sign), check_ffn.py:23-40
E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


# ---------------------------------------------------------------- bf16
def bf16_round(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> nearest-even bf16 -> fp32 (torch's conversion is RNE)."""
    return x.float().to(torch.bfloat16).float()


# ---------------------------------------------------------------- E8M0 codes
def fma_f32(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """fp32 fused multiply-add a * b + c with one rounding (IEEE fmaf, round to nearest even):
    the product of two fp32 values is exact in fp64; the fp64 sum s and its exact error e
    (Knuth's TwoSum) give a * b + c = s + e exactly, and rounding s to fp32 is the single
    rounding of the exact value unless s sits exactly on an fp32 tie, where e's sign decides."""
    a, b, c = (torch.broadcast_to(t.float(), torch.broadcast_shapes(a.shape, b.shape, c.shape)).double().numpy()
               for t in (a, b, c))
    p = a * b
    s = p + c
    bp = s - p
    e = (p - (s - bp)) + (c - bp)
    f = s.astype(np.float32)
    lo = np.nextafter(f, np.float32(-np.inf)).astype(np.float64)
    hi = np.nextafter(f, np.float32(np.inf)).astype(np.float64)
    fd = f.astype(np.float64)
    # s on the midpoint between f and a neighbour: the exact value lies on e's side of it
    go_up = (s == (fd + hi) / 2) & (e > 0)  # s rounded down to f, the exact value is above s
    go_dn = (s == (fd + lo) / 2) & (e < 0)  # s rounded up to f, the exact value is below s
    out = np.where(go_up, np.nextafter(f, np.float32(np.inf)), f)
    out = np.where(go_dn, np.nextafter(f, np.float32(-np.inf)), out)
    return torch.from_numpy(np.ascontiguousarray(out.astype(np.float32)))


def code_ceil(v: torch.Tensor) -> torch.Tensor:
    """Biased exponent of the smallest power of two >= v (v > 0): exponent bits plus one if
    any mantissa bit is set (``mx.py:26-32``, ``check_ffn.py:87-90``). int32."""
    bits = v.float().contiguous().view(torch.int32)
    return ((bits >> 23) & 0xFF) + ((bits & 0x7FFFFF) != 0).int()


def pow2(code: torch.Tensor) -> torch.Tensor:
    """2^(code - 127) in fp32 for integer codes (exact, code 0 included)."""
    return torch.ldexp(torch.ones_like(code, dtype=torch.float32), code.int() - 127)


def mx_mul(code: torch.Tensor) -> torch.Tensor:
    """2^(127 - code) as fp32 for code in [0, 254] (``attention/device.py:84-86``):
    the bit pattern (254 - code) << 23, so code 254 gives 0."""
    return ((254 - code.int()) << 23).view(torch.float32)


# ---------------------------------------------------------------- e4m3 codec (bit level)
def e4m3_encode(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> e4m3fn bytes: clamp to +-448, then torch's round-to-nearest-even conversion
    (the kernels clamp, then convert with satfinite RNE). uint8."""
    return x.float().clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def e4m3_encode_bits(x: torch.Tensor) -> torch.Tensor:
    """``e4m3_encode`` derived independently at the bit level (numpy), to cross-check torch."""
    x = x.float().clamp(-FP8_MAX, FP8_MAX)
    a = np.abs(x.numpy().astype(np.float64))
    sign = (np.signbit(x.numpy())).astype(np.uint8) << 7
    # exponent of the e4m3 binade (normals: 2^-6 .. 2^8; below 2^-6 the subnormal step 2^-9)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.clip(e, -6, 8)
    step = np.ldexp(1.0, (e - 3).astype(np.int64))  # 3 mantissa bits
    q = a / step  # exact: a is fp32, step a power of two
    r = np.rint(q)  # nearest even (np.rint is RNE)
    v = r * step
    # a carry into the next binade is representable as is (the encoding below re-derives it)
    mag = np.zeros_like(a, dtype=np.int64)
    nz = v > 0
    ve = np.floor(np.log2(np.where(nz, v, 1.0)))
    ve = np.clip(ve, -6, 8)
    sub = v < 2.0**-6
    mant_sub = np.rint(v / 2.0**-9).astype(np.int64)  # 0..7
    mant_n = np.rint((v / np.ldexp(1.0, ve.astype(np.int64)) - 1.0) * 8).astype(np.int64)
    exp_n = (ve + 7).astype(np.int64)
    mag = np.where(sub, mant_sub, (exp_n << 3) | mant_n)
    mag = np.where(nz, mag, 0)
    return torch.from_numpy((mag.astype(np.uint8) | sign).astype(np.uint8))


def e4m3_decode(b: torch.Tensor) -> torch.Tensor:
    """e4m3fn bytes -> fp32."""
    b = b.to(torch.int32)
    s = torch.where((b & 0x80) != 0, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = (b & 7).float()
    v = torch.where(e == 0, m * 2.0**-9, torch.ldexp(1.0 + m / 8.0, e - 7))
    return s * v


def e2m1_decode(nib: torch.Tensor) -> torch.Tensor:
    """E2M1 codes (0..15) -> fp32."""
    lut = torch.tensor(E2M1, dtype=torch.float32)
    return lut[nib.long()]


def e2m1_encode(x: torch.Tensor) -> torch.Tensor:
    """fp32 (already divided by its block scale) -> E2M1 code, round to nearest even
    between representable magnitudes, saturating at 6. uint8 codes 0..15."""
    mags = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    a = x.float().abs().clamp(max=6.0)
    d = (a[..., None] - mags).abs()
    best = d.min(-1, keepdim=True).values
    # ties: the candidate with an even mantissa bit (code & 1 == 0)
    cand = (d == best)
    even = torch.tensor([c % 2 == 0 for c in range(8)])
    pick = torch.where(cand & even, 1, 0) * 2 + cand.int()
    code = pick.argmax(-1)
    sign = (x < 0) & (code > 0)
    return (code + 8 * sign.long()).to(torch.uint8)


# ---------------------------------------------------------------- MXFP8 (two scale rules)
def mx_code_vllm(amax: torch.Tensor) -> torch.Tensor:
    """vLLM's ``mxfp8_e4m3_quantize`` code: clamp(code_ceil(RN(max(amax, FLT_MIN) / 448)), 0, 254)
    (``moe.py:232-243``, ``attention/device.py:77-81``)."""
    q = amax.float().clamp_min(FLT_MIN) / FP8_MAX  # IEEE division
    return code_ceil(q).clamp(0, 254)


def mx_code_aiter(amax: torch.Tensor) -> torch.Tensor:
    """aiter's routed-expert code: clamp(code_ceil(max(amax, 1e-10) * RN(1/448)), 1, 254)
    (``moe.py:212-215``, ``check_ffn.py:99``)."""
    q = amax.float().clamp_min(1e-10) * torch.tensor(1.0 / FP8_MAX, dtype=torch.float32)
    return code_ceil(q).clamp(1, 254)


def mxfp8_quant(x: torch.Tensor, rule: str):
    """Per-32 MXFP8 of the last dim: (e4m3 bytes [.., K], codes uint8 [.., K/32])."""
    g = x.float().reshape(*x.shape[:-1], -1, 32)
    amax = g.abs().amax(-1)
    code = mx_code_aiter(amax) if rule == "aiter" else mx_code_vllm(amax)
    inv = mx_mul(code)
    q = e4m3_encode((g * inv[..., None]).clamp(-FP8_MAX, FP8_MAX))
    return q.reshape(x.shape), code.to(torch.uint8)


def mxfp8_dequant(q: torch.Tensor, code: torch.Tensor) -> torch.Tensor:
    v = e4m3_decode(q).reshape(*q.shape[:-1], -1, 32)
    return (v * pow2(code.int())[..., None]).reshape(q.shape)


# ---------------------------------------------------------------- FP8 block-scaled / MXFP4 weights
def deq_fp8_block(w8: torch.Tensor, codes: torch.Tensor, rb: int, cb: int) -> torch.Tensor:
    """e4m3 [N, K] with E8M0 codes per (rb x cb) block -> fp32 (``check_ffn.py:118-121``)."""
    s = pow2(codes.int()).repeat_interleave(rb, 0).repeat_interleave(cb, 1)
    return e4m3_decode(w8) * s[: w8.shape[0], : w8.shape[1]]


def deq_fp4(packed: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
    """[N, K/2] packed E2M1 (even K in the low nibble), [N, K/32] E8M0 -> [N, K] fp32
    (``check_ffn.py:108-115``)."""
    p = packed.to(torch.int32)
    v = torch.stack([e2m1_decode(p & 15), e2m1_decode(p >> 4)], -1).flatten(-2)
    return v * pow2(codes.int()).repeat_interleave(32, -1)


# ---------------------------------------------------------------- deterministic fp64 math
# The kernels' routing scores and router softmax use these instead of the CUDA math
# library so the CPU and the GPU round identically: the same IEEE fp64 operations in
# the same order, no fused multiply-add (the CUDA side uses __dmul_rn / __dadd_rn).
# exp: Cody-Waite reduction x = k ln2 + r, |r| <= ln2/2, then the Taylor series of e^r
# to degree 17 by Horner (truncation < 2^-60 relative). log: x = m 2^e with m in
# [sqrt(1/2), sqrt(2)), log m = 2 atanh(s), s = (m - 1)/(m + 1), the atanh series to
# s^27. log1p(y) = log(u) * y / (u - 1) with u = 1 + y (Goldberg's correction).
LN2_HI = float.fromhex("0x1.62e42fee00000p-1")  # ln 2 to 32 bits: k * LN2_HI is exact
LN2_LO = math.log(2.0) - LN2_HI
INV_LN2 = 1.0 / math.log(2.0)
EXP_COEF = [1.0 / math.factorial(n) for n in range(17, -1, -1)]  # Horner order
ATANH_COEF = [1.0 / (2 * n + 1) for n in range(13, -1, -1)]
LN2 = math.log(2.0)
SQRT_HALF_BITS = 0x3FE6A09E667F3BCD  # sqrt(0.5) as an fp64 bit pattern


def det_exp(x: np.ndarray) -> np.ndarray:
    """e^x for fp64 x in [-700, 700], deterministic (see above)."""
    x = np.asarray(x, dtype=np.float64)
    k = np.rint(x * INV_LN2)
    r = (x - k * LN2_HI) - k * LN2_LO
    p = np.full_like(r, EXP_COEF[0])
    for c in EXP_COEF[1:]:
        p = p * r + c
    # 2^k by bit construction (k within the normal range here)
    two_k = ((k.astype(np.int64) + 1023) << 52).view(np.float64)
    return p * two_k


def det_log(u: np.ndarray) -> np.ndarray:
    """log(u) for fp64 u > 0 normal, deterministic."""
    u = np.asarray(u, dtype=np.float64)
    bits = u.view(np.int64)
    e = (bits >> 52) - 1023
    m_bits = (bits & 0x000FFFFFFFFFFFFF) | 0x3FF0000000000000  # m in [1, 2)
    big = m_bits > (SQRT_HALF_BITS + (1 << 52))  # m > sqrt(2): halve it
    m_bits = np.where(big, m_bits - (1 << 52), m_bits)
    e = np.where(big, e + 1, e)
    m = m_bits.view(np.float64)
    s = (m - 1.0) / (m + 1.0)
    s2 = s * s
    p = np.full_like(s, ATANH_COEF[0])
    for c in ATANH_COEF[1:]:
        p = p * s2 + c
    return e.astype(np.float64) * LN2 + (2.0 * s) * p


def det_softplus(x: np.ndarray) -> np.ndarray:
    """softplus in fp64 for fp32 inputs x <= 20 (``moe.py:305-316`` passes x > 20 through):
    log1p(e^x) with e^x flushed to 0 below x = -700."""
    x = np.asarray(x, dtype=np.float64)
    y = det_exp(np.maximum(x, -700.0))
    u = 1.0 + y
    d = u - 1.0
    safe = np.where(d == 0.0, 1.0, d)
    lg = det_log(u) * (y / safe)
    return np.where(d == 0.0, y, lg)


def route_score(logits: torch.Tensor) -> torch.Tensor:
    """sqrtsoftplus score of fp32 logits: x > 20 -> sqrt(x); else sqrt(fp32(softplus64(x)));
    NaN -> NaN (the caller zeroes it). fp32, bit-exact with the kernel."""
    x = logits.float().numpy()
    with np.errstate(all="ignore"):
        sp = det_softplus(np.where(x > 20.0, 0.0, x)).astype(np.float32)
    sp = np.where(x > 20.0, x, sp).astype(np.float32)
    sp = np.where(np.isnan(x), np.float32(np.nan), sp)
    return torch.from_numpy(np.sqrt(sp).astype(np.float32))
