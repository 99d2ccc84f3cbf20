"""CPU oracle for the routed-expert MoE hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it.  The shipped path runs the CUDA library and fails
loudly when it is missing.

It restates, in numpy, the arithmetic of the reference's MoE layer
(``spark_runtime/lazy_official_runtime.py:980-1002`` ``LazyMoE.forward``) and of
the official DeepSeek ``Gate`` / ``Expert`` / ``act_quant`` / ``fp4_gemm`` /
``fp8_gemm`` that the reference imports at run time
(``spark_runtime/lazy_official_runtime.py:1016-1021``; API exercised in
``scripts/smoke_official_kernels.py:28-51``).  The official ``inference/model.py``
and ``kernel.py`` are a third-party dependency (HF repo
``deepseek-ai/DeepSeek-V4-Flash``, no pinned revision; TileLang 0.1.8 per
``docker/Dockerfile.spark-runtime:4``) that is absent here, so the Gate/Expert
semantics below are the published DeepSeek MoE algorithm with the choices the
benchmark statement fixes (sigmoid scores, correction bias, renormalise,
routed scale), each one documented where it is made.

Pinning:
  * dispatch/combine structure and dtypes: pinned against the reference's own
    ``LazyMoE.forward`` run in the build container (``tests/golden/make_golden.py``);
  * packed-slab format and materialized bytes: pinned against the reference's
    layout builder (``scripts/build_packed_expert_layout.py:76-238``) and its
    C++ loader (``spark_runtime/native/native_packed_loader.cpp``), compiled from
    the reference sources by ``oracle/Makefile``;
  * Gate/Expert arithmetic: parity unpinned at the official-model boundary
    (no golden vectors exist in the reference); the restatement is fixed here.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# ---------------------------------------------------------------------------
# Number formats
# ---------------------------------------------------------------------------

# OCP e2m1: sign | 2-bit exponent (bias 1) | 1-bit mantissa.  Two codes per
# byte, element 2i in the low nibble (torch.float4_e2m1fn_x2 convention; the
# checkpoint stores these bytes as I8, weight-manifest.csv:5510-5512, and the
# runtime reinterprets them, scripts/build_weight_manifest.py:77).
E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)


def _e4m3fn_table() -> np.ndarray:
    """Value of every e4m3fn code: sign | 4-bit exponent (bias 7) | 3-bit mantissa.
    Exponent 15 with mantissa 7 is NaN; there is no infinity; max finite 448."""
    out = np.empty(256, dtype=np.float32)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            out[code] = np.nan
        elif e == 0:
            out[code] = s * (m / 8.0) * 2.0 ** -6
        else:
            out[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return out


E4M3_VALUES = _e4m3fn_table()
_E4M3_POS = E4M3_VALUES[:127].astype(np.float64)  # codes 0x00..0x7E, increasing
E4M3_MAX = 448.0


def e8m0_to_f32(code: np.ndarray) -> np.ndarray:
    """ue8m0 scale byte b -> 2**(b-127) (b == 255 is NaN in the OCP MX spec)."""
    code = np.asarray(code, dtype=np.int32)
    out = np.ldexp(np.float32(1.0), code - 127).astype(np.float32)
    return np.where(code == 255, np.float32(np.nan), out)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = np.where(nan, (u >> 16) | 0x40, rounded)
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (ties to even), kept as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def f32_to_e4m3_codes(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn code, round to nearest even, saturating to +-448.

    Same result as the PTX ``cvt.rn.satfinite.e4m3x2.f32`` conversion for
    finite inputs.  The sign of zero is kept (a negative value that rounds to
    zero gives 0x80)."""
    x = np.asarray(x, dtype=np.float32)
    neg = np.signbit(x)
    a = np.minimum(np.abs(x).astype(np.float64), E4M3_MAX)
    # quantum: 2^(e-3) in the normal range (e = floor(log2 a) >= -6), 2^-9 below
    _, ex = np.frexp(a)  # a = m * 2^ex, m in [0.5, 1)
    e = np.maximum(ex - 1, -6)
    q = np.ldexp(1.0, e - 3)
    r = np.rint(a / q) * q  # np.rint: round half to even; a/q exact
    code = np.searchsorted(_E4M3_POS, r).astype(np.uint8)
    return np.where(neg, code | 0x80, code).astype(np.uint8)


def decode_e4m3(codes: np.ndarray) -> np.ndarray:
    return E4M3_VALUES[np.asarray(codes, dtype=np.uint8)]


# byte -> (low nibble value, high nibble value): one lookup per packed byte
_E2M1_PAIRS = np.stack([E2M1_VALUES[np.arange(256) & 0xF], E2M1_VALUES[np.arange(256) >> 4]], axis=1)


def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    """[..., K/2] bytes -> [..., K] fp32, low nibble first."""
    packed = np.asarray(packed, dtype=np.uint8)
    return _E2M1_PAIRS[packed].reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def dequant_fp4_weight(packed: np.ndarray, scale: np.ndarray, block: int = 32) -> np.ndarray:
    """FP4 e2m1 [N, K/2] bytes with ue8m0 scales [N, K/block] -> fp32 [N, K].
    Exact: every product is representable in fp32 (and in bf16), so the
    multi-threaded torch CPU lookup and multiply below give the same bits as
    the element-wise definition (unpack_e2m1 x 2^(scale-127))."""
    import torch

    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    n = packed.shape[0]
    w = torch.from_numpy(_E2M1_PAIRS)[torch.from_numpy(packed).long()].reshape(n, -1)
    s = torch.from_numpy(np.ascontiguousarray(e8m0_to_f32(scale), dtype=np.float32))
    k = w.shape[1]
    return (w.view(n, k // block, block) * s[:, :, None]).view(n, k).numpy()


def dequant_fp8_weight(codes: np.ndarray, scale: np.ndarray, block: int = 128) -> np.ndarray:
    """FP8 e4m3 [N, K] with ue8m0 block scales [N/block, K/block] -> fp32 [N, K]."""
    w = decode_e4m3(codes)
    s = e8m0_to_f32(scale)
    s_full = np.repeat(np.repeat(s, block, axis=0), block, axis=1)
    return (w * s_full[: w.shape[0], : w.shape[1]]).astype(np.float32)


# ---------------------------------------------------------------------------
# act_quant: official kernel.act_quant(x, 128, "ue8m0") semantics
# ---------------------------------------------------------------------------

_INV_E4M3_MAX = np.float32(1.0) / np.float32(448.0)


def ceil_log2_exact(v: np.ndarray) -> np.ndarray:
    """ceil(log2(v)) for positive normal fp32 v, computed exactly from the bits."""
    m, ex = np.frexp(np.asarray(v, dtype=np.float32))
    return np.where(m == 0.5, ex - 1, ex).astype(np.int32)


def act_quant(x: np.ndarray, block: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """bf16 activations (given as fp32 values) [M, K] -> (e4m3 codes [M, K],
    ue8m0 scale bytes [M, K/block]).

    Per block: amax = max(|x|, 1e-4); s = 2^ceil(log2(amax * (1/448))) (a power
    of two, the ``ue8m0`` scale format of the checkpoint's quantization_config,
    results/spark-66c9/checkpoint-inventory.summary.json ``scale_fmt``);
    q = e4m3(x / s).  Since amax/s <= 448 nothing saturates."""
    x = np.asarray(x, dtype=np.float32)
    M, K = x.shape
    assert K % block == 0
    xb = x.reshape(M, K // block, block)
    amax = np.max(np.abs(xb), axis=-1)
    amax = np.maximum(amax, np.float32(1e-4))
    v = (amax * _INV_E4M3_MAX).astype(np.float32)
    e = ceil_log2_exact(v)
    q = f32_to_e4m3_codes(np.ldexp(xb, -e[..., None]).astype(np.float32))
    return q.reshape(M, K), (e + 127).astype(np.uint8)


# e2m1 magnitudes by code, and the rounding boundaries between neighbouring
# codes: a magnitude exactly on a boundary rounds to the even code (down at
# 0.25, 1.25, 2.5, 5; up at 0.75, 1.75, 3.5); above 5 it saturates to 6.
_E2M1_DOWN_TIES = np.array([0.25, 1.25, 2.5, 5.0], np.float32)
_E2M1_UP_TIES = np.array([0.75, 1.75, 3.5], np.float32)
_INV_E2M1_MAX = np.float32(1.0 / 6.0)


def f32_to_e2m1_codes(v: np.ndarray) -> np.ndarray:
    """fp32 -> 4-bit e2m1 codes (sign in bit 3), round to nearest even,
    saturating at +-6 (cvt.rn.satfinite semantics)."""
    v = np.asarray(v, np.float32)
    a = np.abs(v)
    code = (a[..., None] > _E2M1_DOWN_TIES).sum(-1) + (a[..., None] >= _E2M1_UP_TIES).sum(-1)
    return (code.astype(np.uint8) | (np.signbit(v).astype(np.uint8) << 3)).astype(np.uint8)


def fp4_act_quant(x: np.ndarray, block: int = 32) -> tuple[np.ndarray, np.ndarray]:
    """The official ``fp4_act_quant(x, 32)`` (scripts/smoke_official_kernels.py:
    32-34; result types torch.float4_e2m1fn_x2 codes and float8_e8m0fnu scales,
    docs/experiments/016-native-kernel-smoke.md:50), restated with the
    conventions of ``act_quant``: per block of 32, amax = max(|x|, 1e-4),
    s = 2^ceil(log2(amax * fp32(1/6))), q = e2m1(x / s) with round to nearest
    even; codes packed two per byte, element 2i in the low nibble.
    Returns (packed [M, K/2] uint8, scale bytes [M, K/block] uint8)."""
    x = np.asarray(x, dtype=np.float32)
    M, K = x.shape
    assert K % block == 0 and block % 2 == 0
    xb = x.reshape(M, K // block, block)
    amax = np.maximum(np.max(np.abs(xb), axis=-1), np.float32(1e-4))
    e = ceil_log2_exact((amax * _INV_E2M1_MAX).astype(np.float32))
    codes = f32_to_e2m1_codes(np.ldexp(xb, -e[..., None]).astype(np.float32)).reshape(M, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, (e + 127).astype(np.uint8)


def fp4_act_dequant(packed: np.ndarray, s: np.ndarray, block: int = 32) -> np.ndarray:
    vals = unpack_e2m1(packed)
    return (vals * np.repeat(e8m0_to_f32(s), block, axis=1)).astype(np.float32)


def act_dequant(q: np.ndarray, s: np.ndarray, block: int = 128) -> np.ndarray:
    vals = decode_e4m3(q)
    return (vals * np.repeat(e8m0_to_f32(s), block, axis=1)).astype(np.float32)


# ---------------------------------------------------------------------------
# Canonical fp32 sigmoid (bit-exact twin of the device routine)
# ---------------------------------------------------------------------------
# exp() by Cody & Waite range reduction (two-constant split of ln 2 as in
# Moshier's Cephes expf: C1 = 355/512, C2 = -2.12194440e-4) followed by the
# degree-7 Taylor polynomial of e^r on |r| <= ln(2)/2 in Horner form.  Every
# step is one IEEE fp32 operation rounded to nearest even with no fused
# multiply-add, so the CUDA routine (which uses __fmul_rn/__fadd_rn/__fdiv_rn)
# produces the same bits.  Relative error vs. the true exp is < 2e-7.

_F = np.float32
_LOG2E = _F(1.4426950408889634)
_C1 = _F(0.693359375)
_C2 = _F(-2.12194440e-4)
_TAYLOR = [_F(1.0 / 5040.0), _F(1.0 / 720.0), _F(1.0 / 120.0), _F(1.0 / 24.0),
           _F(1.0 / 6.0), _F(0.5), _F(1.0), _F(1.0)]
SIGMOID_CLAMP = _F(80.0)


def exp_canonical(t: np.ndarray) -> np.ndarray:
    t = np.asarray(t, dtype=np.float32)
    n = np.rint((t * _LOG2E).astype(np.float32)).astype(np.float32)
    r = (t - (n * _C1).astype(np.float32)).astype(np.float32)
    r = (r - (n * _C2).astype(np.float32)).astype(np.float32)
    p = np.full_like(r, _TAYLOR[0])
    for c in _TAYLOR[1:]:
        p = ((p * r).astype(np.float32) + c).astype(np.float32)
    return np.ldexp(p, n.astype(np.int32)).astype(np.float32)


def sigmoid_canonical(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    t = np.clip(-x, -SIGMOID_CLAMP, SIGMOID_CLAMP).astype(np.float32)
    e = exp_canonical(t)
    return (_F(1.0) / (_F(1.0) + e).astype(np.float32)).astype(np.float32)


# ---------------------------------------------------------------------------
# Gate (official Gate.forward(x, input_ids) -> (weights[T,k], indices[T,k]),
# called at lazy_official_runtime.py:983)
# ---------------------------------------------------------------------------

def gate_logits(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """logits[t, e] = sum_h x[t,h] * W[e,h]; accumulated in float64 then rounded
    to fp32 (the device accumulates in fp32, so logits agree to ~1e-6 rel)."""
    return (np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32)


def route_from_logits(logits: np.ndarray, bias: np.ndarray | None, topk: int,
                      route_scale: float) -> tuple[np.ndarray, np.ndarray]:
    """sigmoid scores; top-k of (score + bias), descending, ties to the lower
    expert id; weights = scores at the chosen ids, renormalised to sum 1
    (summed in rank order), times route_scale.  All fp32, bit-exact."""
    scores = sigmoid_canonical(logits)
    sel = scores if bias is None else (scores + np.asarray(bias, np.float32)).astype(np.float32)
    order = np.argsort(-sel, axis=-1, kind="stable")  # stable: lower id first on ties
    idx = order[:, :topk]
    wts = np.take_along_axis(scores, idx, axis=-1).astype(np.float32)
    total = wts[:, 0].copy()
    for j in range(1, topk):
        total = (total + wts[:, j]).astype(np.float32)
    wts = (wts / total[:, None]).astype(np.float32)
    wts = (wts * np.float32(route_scale)).astype(np.float32)
    return wts, idx.astype(np.int64)


def routing_flips(device_indices: np.ndarray, logits_ref: np.ndarray, bias: np.ndarray | None,
                  topk: int) -> list[tuple[int, float]]:
    """Tokens whose device top-k set differs from the top-k the oracle selects
    on its own (float64-accumulated) logits, with the score gap of each flip:
    (token, gap relative to the boundary score), where the gap is how far the
    oracle's best rejected-by-the-device expert beats the device's worst
    choice that the oracle rejected, in selection score (sigmoid + bias).  A
    flip is legitimate only when that gap is within the logits' accumulation
    error (a near tie)."""
    scores = sigmoid_canonical(np.asarray(logits_ref, np.float32))
    sel = scores if bias is None else (scores + np.asarray(bias, np.float32)).astype(np.float32)
    order = np.argsort(-sel, axis=-1, kind="stable")[:, :topk]
    out = []
    for t in range(device_indices.shape[0]):
        d, r = set(device_indices[t].tolist()), set(order[t].tolist())
        if d == r:
            continue
        only_r = sorted(r - d)
        only_d = sorted(d - r)
        gap = float(max(sel[t, e] for e in only_r) - min(sel[t, e] for e in only_d))
        boundary = float(abs(sel[t, order[t, topk - 1]])) or 1e-30
        out.append((t, gap / boundary))
    return out


def hash_route(logits: np.ndarray, tid2eid: np.ndarray, input_ids: np.ndarray, route_scale: float):
    """Hash-routed layers (gate.tid2eid [vocab, k], weight-manifest.csv:3; the
    official Gate's hash mode is absent here, so this is the restated choice):
    experts = tid2eid[input_id] in row order; weights = their canonical
    sigmoid scores renormalised to sum 1 in row order (fp32), x route_scale."""
    idx = np.asarray(tid2eid)[np.asarray(input_ids).reshape(-1)].astype(np.int64)
    T, k = idx.shape
    scores = sigmoid_canonical(np.asarray(logits, np.float32))
    w = scores[np.arange(T)[:, None], idx].astype(np.float32)
    total = w[:, 0].copy()
    for j in range(1, k):
        total = (total + w[:, j]).astype(np.float32)
    w = ((w / total[:, None]).astype(np.float32) * np.float32(route_scale)).astype(np.float32)
    return w, idx


def gate_forward(x, w, bias, topk, route_scale):
    logits = gate_logits(x, w)
    wts, idx = route_from_logits(logits, bias, topk, route_scale)
    return wts, idx, logits


# ---------------------------------------------------------------------------
# Expert (official Expert(dim, inter, dtype=, swiglu_limit=).forward(x, weights))
# ---------------------------------------------------------------------------

@dataclass
class ExpertWeights:
    """One expert's parameters in checkpoint format.

    Routed (fp4): w1/w3 [I, H/2] e2m1x2 bytes, scale [I, H/32]; w2 [H, I/2],
    scale [H, I/32] (weight-manifest.csv:4731-4733,5510-5512).
    Shared (fp8): w1/w3 [I, H] e4m3 codes, scale [I/128, H/128]; w2 [H, I],
    scale [H/128, I/128] (weight-manifest.csv:5499-5509)."""
    w1: np.ndarray
    w1_scale: np.ndarray
    w2: np.ndarray
    w2_scale: np.ndarray
    w3: np.ndarray
    w3_scale: np.ndarray
    fp4: bool = True

    def dense(self):
        if self.fp4:
            f = dequant_fp4_weight
        else:
            f = dequant_fp8_weight
        return f(self.w1, self.w1_scale), f(self.w2, self.w2_scale), f(self.w3, self.w3_scale)


def quantized_linear(x_bf16: np.ndarray, w_dense: np.ndarray) -> np.ndarray:
    """official ``linear`` for a low-precision weight: act_quant(x, 128, ue8m0)
    then fp4_gemm / fp8_gemm -> bf16 (kernel API per
    scripts/smoke_official_kernels.py:36-50).  Products are exact; the dot
    product is accumulated in float64 and rounded once (device: fp32 tensor-core
    accumulation), then the result is rounded to bf16."""
    q, s = act_quant(x_bf16)
    return dequant_linear(act_dequant(q, s), w_dense)


def dequant_linear(a: np.ndarray, w_dense: np.ndarray) -> np.ndarray:
    """The GEMM of ``quantized_linear`` on already quantized-and-dequantized
    activations ``a``.  Every product of an e4m3 activation and an e2m1 / e4m3
    weight (with power-of-two scales) has at most 5 significant bits and the
    exponents of one dot product span far fewer than float64's 53 bits, so the
    float64 sum is exact whatever the summation order; the multi-threaded torch
    CPU product therefore gives the bits of a sequential float64 sum."""
    import torch

    a64 = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).double()
    w64 = torch.from_numpy(np.ascontiguousarray(w_dense, dtype=np.float32)).double()
    return round_bf16((a64 @ w64.T).numpy().astype(np.float32))


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1.0) + np.exp(-x.astype(np.float64)).astype(np.float32))).astype(np.float32)


def expert_forward(x_bf16: np.ndarray, ew: ExpertWeights, route_w: np.ndarray | None,
                   swiglu_limit: float, dense=None, fp4_act: bool = False) -> np.ndarray:
    """SwiGLU expert.  g = w1(x), u = w3(x) (bf16 outputs); if swiglu_limit > 0:
    u = clamp(u, -limit, limit), g = min(g, limit); h = silu(g) * u, times the
    routing weight when given (applied before w2, in fp32); h is cast to bf16
    and fed through w2.  Returns bf16 values as fp32 [n, H].

    fp4_act: x and h are quantized by fp4_act_quant (e2m1, per-32 scales)
    instead of act_quant for w1 / w3 and for w2 (the library's opt-in
    FP4-activation mode); the products stay exact in float64 (e2m1 x e2m1
    with power-of-two scales)."""
    if fp4_act:
        q, s = fp4_act_quant(x_bf16)
        return expert_forward_dequant(fp4_act_dequant(q, s), ew, route_w, swiglu_limit, dense, fp4_h=True)
    q, s = act_quant(x_bf16)
    return expert_forward_dequant(act_dequant(q, s), ew, route_w, swiglu_limit, dense)


def expert_forward_dequant(a: np.ndarray, ew: ExpertWeights, route_w: np.ndarray | None,
                           swiglu_limit: float, dense=None, fp4_h: bool = False) -> np.ndarray:
    """``expert_forward`` from the dequantized act_quant of its input (the form
    in which an expert-parallel rank receives the rows).  fp4_h: h goes through
    fp4_act_quant (per 32) instead of act_quant before w2."""
    w1, w2, w3 = dense if dense is not None else ew.dense()
    g = dequant_linear(a, w1)
    u = dequant_linear(a, w3)
    if swiglu_limit and swiglu_limit > 0:
        lim = np.float32(swiglu_limit)
        u = np.clip(u, -lim, lim)
        g = np.minimum(g, lim)
    h = (silu(g) * u).astype(np.float32)
    if route_w is not None:
        h = (h * np.asarray(route_w, np.float32).reshape(-1, 1)).astype(np.float32)
    if fp4_h:
        q, s = fp4_act_quant(round_bf16(h))
        return dequant_linear(fp4_act_dequant(q, s), w2)
    return quantized_linear(round_bf16(h), w2)


# ---------------------------------------------------------------------------
# MoE layer (LazyMoE.forward, lazy_official_runtime.py:980-1002)
# ---------------------------------------------------------------------------

@dataclass
class MoEWeights:
    gate_w: np.ndarray            # [E, H] fp32 values (bf16 or fp32 checkpoint)
    gate_bias: np.ndarray | None  # [E] fp32
    experts: list                 # list[ExpertWeights], routed
    shared: ExpertWeights         # fp8 shared expert
    topk: int
    route_scale: float
    swiglu_limit: float


def combine(T: int, H: int, indices: np.ndarray, expert_out: dict, shared_out: np.ndarray,
            e_begin: int = 0, e_end: int | None = None) -> np.ndarray:
    """y = 0 (fp32); for each active expert in ascending id: y[rows] += out_e;
    then y += shared; cast to bf16 (lazy_official_runtime.py:984,995-1002)."""
    y = np.zeros((T, H), dtype=np.float32)
    E = e_end
    for e in sorted(expert_out):
        if e < e_begin or (E is not None and e >= E):
            continue
        rows = expert_out[e][0]
        y[rows] = (y[rows] + expert_out[e][1]).astype(np.float32)
    y = (y + shared_out).astype(np.float32)
    return round_bf16(y)


def moe_forward(x_bf16: np.ndarray, mw: MoEWeights, routing=None, dense_cache=None, workers: int = 1,
                fp4_act: bool = False):
    """Full layer.  ``routing`` = (weights, indices) overrides the gate (used to
    check the expert math on the device's own routing).  Returns
    (y bf16-as-fp32 [T,H], weights, indices, per-route outputs dict).

    ``workers`` > 1 evaluates the experts in a thread pool (the weight decode
    and the float64 products release the GIL); each expert's output is the
    same either way and the combine always sums in ascending expert id.

    ``fp4_act``: the routed experts take FP4 activations for w1 / w3 (see
    ``expert_forward``); the shared expert keeps act_quant, as the library's
    FP4-activation mode does."""
    T, H = x_bf16.shape
    if routing is None:
        wts, idx, _ = gate_forward(x_bf16, mw.gate_w, mw.gate_bias, mw.topk, mw.route_scale)
    else:
        wts, idx = routing

    def one(e):
        rows, top = np.nonzero(idx == e)  # torch.where order: row-major
        dense = dense_cache(e) if dense_cache is not None else None
        return e, (rows, expert_forward(x_bf16[rows], mw.experts[e], wts[rows, top], mw.swiglu_limit, dense,
                                        fp4_act=fp4_act))

    active = [int(e) for e in np.unique(idx)]
    if workers > 1 and len(active) > 1:
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(workers) as pool:
            outs = dict(pool.map(one, active))
    else:
        outs = dict(one(e) for e in active)
    shared_dense = dense_cache("shared") if dense_cache is not None else None
    sh = expert_forward(x_bf16, mw.shared, None, mw.swiglu_limit, shared_dense)
    y = combine(T, H, idx, outs, sh)
    return y, wts, idx, outs


def route_plan(indices: np.ndarray, n_experts: int, block_n: int, shared_rows: int, align: int = 32):
    """Segment layout of the routes (the dispatch of lazy_official_runtime.py:985,996-998).

    Expert e's rows are the tokens ``torch.where(indices == e)`` returns, in that
    (token) order; segments are the experts in ascending id followed by the
    shared expert (the first ``shared_rows`` tokens), each padded to ``align``
    rows.  Returns dict(counts [E+1], seg_start [E+2], route_slot [T*k] (-1 for
    a skipped route), slot_token [rows] (-1 on padding), tiles [(segment,
    row0, rows)]).  Indices of -1 are skipped routes."""
    idx = np.asarray(indices).reshape(indices.shape[0], -1)
    T, k = idx.shape
    flat = idx.reshape(-1)
    counts = np.zeros(n_experts + 1, dtype=np.int64)
    seg_start = np.zeros(n_experts + 2, dtype=np.int64)
    route_slot = np.full(T * k, -1, dtype=np.int64)
    members = []
    for e in range(n_experts):
        rows, top = np.nonzero(idx == e)
        members.append(rows * k + top)
        counts[e] = rows.size
    counts[n_experts] = shared_rows
    run = 0
    for s in range(n_experts + 1):
        seg_start[s] = run
        run += -(-int(counts[s]) // align) * align
    seg_start[n_experts + 1] = run
    slot_token = np.full(run, -1, dtype=np.int64)
    for e in range(n_experts):
        slots = seg_start[e] + np.arange(counts[e])
        route_slot[members[e]] = slots
        slot_token[slots] = members[e] // k
    slot_token[seg_start[n_experts]:seg_start[n_experts] + shared_rows] = np.arange(shared_rows)
    tiles = [(s, int(seg_start[s]) + m, min(block_n, int(counts[s]) - m))
             for s in range(n_experts + 1) for m in range(0, int(counts[s]), block_n)]
    return {"counts": counts, "seg_start": seg_start, "route_slot": route_slot, "slot_token": slot_token,
            "tiles": tiles}


def moe_forward_ep(x_bf16_per_rank: list, mw: MoEWeights, world: int, routing_per_rank=None):
    """Expert-parallel layer: every rank routes its own tokens; rank r owns
    experts [r*E/W, (r+1)*E/W) (lazy_official_runtime.py:956-965).  Each token's
    result is the sum over its routes of the owning ranks' outputs plus its own
    shared-expert output, i.e. the same value as the single-GPU layer."""
    res = []
    for r, x in enumerate(x_bf16_per_rank):
        routing = None if routing_per_rank is None else routing_per_rank[r]
        res.append(moe_forward(x, mw, routing)[0])
    return res


# ---------------------------------------------------------------------------
# Expert parallelism: dispatch / owning-rank forward / combine.  Rank r owns
# experts [r*E/W, (r+1)*E/W) (lazy_official_runtime.py:956-965); instead of
# replicating tokens and all-reducing y (:999-1000), each token's act_quant
# row travels once to every rank owning one of its experts and every route's
# bf16 output row travels back.  Row format (one send row):
#   [0,H) e4m3 codes | [H,H+H/128) ue8m0 scale bytes |
#   k x {int32 expert (-1 = another rank's), f32 weight, int32 return index}
#   | zero padding to a multiple of 16 bytes.
# ---------------------------------------------------------------------------
EP_META = np.dtype([("e", "<i4"), ("w", "<f4"), ("r", "<i4")])


def ep_row_bytes(hidden: int, topk: int) -> int:
    return -(-(hidden + hidden // 128 + EP_META.itemsize * topk) // 16) * 16


def ep_dispatch(x_bf16: np.ndarray, weights: np.ndarray, indices: np.ndarray, n_experts: int, world: int):
    """-> (send [rows, row_bytes] u8, send_counts [world, 2] (rows, routes), ret_pos [T, k]).

    Rows for rank d follow those for ranks < d; inside, tokens in order.  A
    route's return index counts the routes to rank d in token order, then k
    order; ret_pos adds the routes to earlier ranks."""
    x = np.asarray(x_bf16, np.float32)
    T, H = x.shape
    k = indices.shape[1]
    per = n_experts // world
    dst = np.asarray(indices) // per
    q, s = act_quant(x) if T else (np.zeros((0, H), np.uint8), np.zeros((0, H // 128), np.uint8))
    rows = [(d, t, [j for j in range(k) if dst[t, j] == d]) for d in range(world) for t in range(T)]
    rows = [r for r in rows if r[2]]
    counts = np.zeros((world, 2), np.int32)
    for d, _, js in rows:
        counts[d, 0] += 1
        counts[d, 1] += len(js)
    route_base = np.concatenate([[0], np.cumsum(counts[:, 1])[:-1]]).astype(np.int64)
    rb = ep_row_bytes(H, k)
    send = np.zeros((len(rows), rb), np.uint8)
    ret_pos = np.full((T, k), -1, np.int32)
    nxt = np.zeros(world, np.int64)
    for n, (d, t, js) in enumerate(rows):
        send[n, :H] = q[t]
        send[n, H:H + H // 128] = s[t]
        meta = np.zeros(k, EP_META)
        meta["e"], meta["r"] = -1, -1
        for j in js:
            meta[j] = (indices[t, j], weights[t, j], nxt[d])
            ret_pos[t, j] = route_base[d] + nxt[d]
            nxt[d] += 1
        send[n, H + H // 128:H + H // 128 + EP_META.itemsize * k] = meta.view(np.uint8)
    return send, counts, ret_pos


def ep_expert_forward(mw: MoEWeights, n_experts: int, rank: int, world: int, x_own: np.ndarray,
                      recv: np.ndarray, recv_counts: np.ndarray, dense_cache=None):
    """Owning rank: every received route's output row, placed in the return
    buffer (blocks by source rank, return index inside), and the shared
    expert over this rank's own tokens.  -> (ret_send [routes, H], shared [T_own, H])."""
    H = np.asarray(x_own).shape[1]
    k = mw.topk
    per = n_experts // world
    n_routes = int(np.sum(recv_counts[:, 1]))
    ret = np.zeros((n_routes, H), np.float32)
    src_of_row = np.repeat(np.arange(world), recv_counts[:, 0])
    route_base = np.concatenate([[0], np.cumsum(recv_counts[:, 1])[:-1]]).astype(np.int64)
    R = recv.shape[0]
    if R:
        meta = np.ascontiguousarray(recv[:, H + H // 128:H + H // 128 + EP_META.itemsize * k]).view(EP_META)
        a = act_dequant(recv[:, :H], recv[:, H:H + H // 128])
        for e in sorted(set(int(v) for v in meta["e"].reshape(-1) if v >= 0)):
            assert rank * per <= e < (rank + 1) * per, "route sent to the wrong rank"
            rows, top = np.nonzero(meta["e"] == e)
            dense = dense_cache(e) if dense_cache is not None else None
            out = expert_forward_dequant(a[rows], mw.experts[e], meta["w"][rows, top], mw.swiglu_limit, dense)
            ret[route_base[src_of_row[rows]] + meta["r"][rows, top]] = out
    shared_dense = dense_cache("shared") if dense_cache is not None else None
    x_own = np.asarray(x_own, np.float32)
    shared = (expert_forward(x_own, mw.shared, None, mw.swiglu_limit, shared_dense) if x_own.shape[0]
              else np.zeros((0, H), np.float32))
    return ret, shared


def ep_combine(ret_recv: np.ndarray, ret_pos: np.ndarray, indices: np.ndarray, shared: np.ndarray) -> np.ndarray:
    """y[t] = bf16( sum over t's routes in ascending expert id of ret_recv[ret_pos] + shared[t] )."""
    T, k = indices.shape
    y = np.zeros((T, shared.shape[1]), np.float32)
    for t in range(T):
        for j in np.argsort(indices[t], kind="stable"):
            y[t] = (y[t] + ret_recv[ret_pos[t, j]]).astype(np.float32)
    return round_bf16((y + shared).astype(np.float32))


# ---------------------------------------------------------------------------
# Packed slab / arena (scripts/build_packed_expert_layout.py:76-86,179-215;
# lazy_official_runtime.py:761-917; native_packed_loader.cpp:199-321)
# ---------------------------------------------------------------------------

# Tensor order inside one packed expert block (tensor_sort_key, :76-86).
PACKED_ORDER = ("w1.scale", "w2.scale", "w3.scale", "w1.weight", "w2.weight", "w3.weight")


def expert_block_layout(hidden: int, inter: int) -> list[tuple[str, int, int]]:
    """(name, offset, bytes) of the six routed-expert tensors in a packed block."""
    sizes = {
        "w1.scale": inter * hidden // 32,
        "w2.scale": hidden * inter // 32,
        "w3.scale": inter * hidden // 32,
        "w1.weight": inter * hidden // 2,
        "w2.weight": hidden * inter // 2,
        "w3.weight": inter * hidden // 2,
    }
    out, off = [], 0
    for name in PACKED_ORDER:
        out.append((name, off, sizes[name]))
        off += sizes[name]
    return out


def materialize_block(block: bytes | np.ndarray, hidden: int, inter: int) -> dict[str, np.ndarray]:
    """Planned slice copies of one packed block into its six parameters
    (ExpertCopyPlan::copy_storage_to_tensors, native_packed_loader.cpp:199-230)."""
    buf = np.frombuffer(bytes(block), dtype=np.uint8) if not isinstance(block, np.ndarray) else block
    return {name: buf[off:off + n].copy() for name, off, n in expert_block_layout(hidden, inter)}


def decode_block_bf16(block: np.ndarray, hidden: int, inter: int) -> dict[str, np.ndarray]:
    """Exact e2m1 x ue8m0 -> bf16 decode of w1/w2/w3 (bf16 bit patterns)."""
    p = materialize_block(block, hidden, inter)
    out = {}
    for w, (n, k) in (("w1", (inter, hidden)), ("w2", (hidden, inter)), ("w3", (inter, hidden))):
        dense = dequant_fp4_weight(p[f"{w}.weight"].reshape(n, k // 2), p[f"{w}.scale"].reshape(n, k // 32))
        out[w] = f32_to_bf16_bits(dense)
    return out


def sf_atoms(scale_rows: np.ndarray) -> np.ndarray:
    """Tensor-memory scale-factor atoms for a [N, K/32] ue8m0 matrix.

    One 512-byte atom per (128-row block nb, 128-column K tile kt), stored
    (nb, kt) row-major; inside an atom row m of the block and scale b (0..3) of
    the tile sit at byte (m % 32) * 16 + (m // 32) * 4 + b.  This is the
    32-lane x 128-bit source layout of tcgen05.cp .32x128b.warpx4."""
    s = np.asarray(scale_rows, dtype=np.uint8)
    N, KS = s.shape
    NB, KT = (N + 127) // 128, KS // 4
    pad = np.zeros((NB * 128, KS), dtype=np.uint8)
    pad[:N] = s
    v = pad.reshape(NB, 4, 32, KT, 4)          # nb, m1, m0, kt, b
    return np.ascontiguousarray(v.transpose(0, 3, 2, 1, 4)).reshape(-1)  # nb, kt, m0, m1, b


def sf_atoms_fp8(scale_blocks: np.ndarray, n_rows: int, k: int) -> np.ndarray:
    """Atoms for an fp8 weight with [N/128, K/128] block scales: every per-32
    scale of a row is its 128x128 block's scale."""
    s = np.asarray(scale_blocks, dtype=np.uint8)
    full = np.repeat(np.repeat(s, 128, axis=0)[:n_rows], 4, axis=1)[:, : k // 32]
    return sf_atoms(full)


# ---------------------------------------------------------------------------
# Adapters from the packed formats to the oracle's structures
# ---------------------------------------------------------------------------

def expert_from_block(block: np.ndarray, hidden: int, inter: int) -> ExpertWeights:
    """Routed expert parameters from one packed block (packed slab order)."""
    p = materialize_block(np.asarray(block, dtype=np.uint8), hidden, inter)
    return ExpertWeights(
        w1=p["w1.weight"].reshape(inter, hidden // 2), w1_scale=p["w1.scale"].reshape(inter, hidden // 32),
        w2=p["w2.weight"].reshape(hidden, inter // 2), w2_scale=p["w2.scale"].reshape(hidden, inter // 32),
        w3=p["w3.weight"].reshape(inter, hidden // 2), w3_scale=p["w3.scale"].reshape(inter, hidden // 32),
        fp4=True)


def shared_from_tensors(t: dict) -> ExpertWeights:
    """fp8 shared expert from {w1.weight, w1.scale, ...} uint8 arrays."""
    a = {k: np.asarray(v, dtype=np.uint8) for k, v in t.items()}
    return ExpertWeights(w1=a["w1.weight"], w1_scale=a["w1.scale"], w2=a["w2.weight"], w2_scale=a["w2.scale"],
                         w3=a["w3.weight"], w3_scale=a["w3.scale"], fp4=False)
