"""The oracle's restatement of the official fp4_act_quant(x, 32) (CPU):
e2m1 rounding to nearest even with saturation, the per-32 power-of-two scale,
nibble packing, and the FP4-activation expert (x and h quantized per 32)
against a dense float64 reference of the same quantized operands."""

import numpy as np

from oracle import moe_oracle as O


def test_e2m1_rounding_ties_and_saturation():
    v = np.array([0.0, 0.2, 0.25, 0.26, 0.75, 1.25, 1.3, 1.75, 2.5, 2.6, 3.5, 5.0, 5.1, 6.0, 100.0,
                  -0.0, -0.25, -1.75, -7.0], np.float32)
    want = [0.0, 0.0, 0.0, 0.5, 1.0, 1.0, 1.5, 2.0, 2.0, 3.0, 4.0, 4.0, 6.0, 6.0, 6.0,
            -0.0, -0.0, -2.0, -6.0]
    got = O.E2M1_VALUES[O.f32_to_e2m1_codes(v)]
    assert np.array_equal(got, np.array(want, np.float32))
    assert np.array_equal(np.signbit(got), np.signbit(np.array(want, np.float32)))


def test_fp4_act_quant_scale_packing_and_bound():
    g = np.random.default_rng(3)
    x = (g.standard_normal((5, 256)) * np.array([1e-6, 0.1, 1.0, 30.0, 1e4])[:, None]).astype(np.float32)
    x[0, :32] = 0.0
    x[1, 32:64] = 0.0
    x[1, 40] = 6.0 * 2.0 ** -3          # amax / 6 exactly a power of two
    q, s = O.fp4_act_quant(x)
    assert q.shape == (5, 128) and s.shape == (5, 8) and q.dtype == np.uint8
    assert s[1, 1] == 127 - 3            # no rounding up at an exact power of two
    assert s[0, 0] == 127 + int(np.ceil(np.log2(1e-4 / 6)))  # amax floored at 1e-4
    # element 2i in the low nibble
    codes = O.f32_to_e2m1_codes(np.ldexp(x[2, :2], -(s[2, 0].astype(int) - 127)))
    assert q[2, 0] == (codes[0] | (codes[1] << 4))
    d = O.fp4_act_dequant(q, s)
    blocks = np.abs(x).reshape(5, 8, 32).max(-1)
    # at most half the widest grid step (4 -> 6) times the block scale, and the
    # scale is below 2 amax / 6
    err = np.abs(d - x).reshape(5, 8, 32).max(-1)
    scale = O.e8m0_to_f32(s)
    assert np.all(err <= scale) and np.all(scale < 2 * np.maximum(blocks, 1e-4) / 6)


def test_fp4_activation_expert_against_dense_reference():
    H, I, n = 256, 128, 5
    g = np.random.default_rng(4)
    x = O.round_bf16(g.standard_normal((n, H)).astype(np.float32))
    w1, w2, w3 = (g.standard_normal(s).astype(np.float32) * 0.05 for s in ((I, H), (H, I), (I, H)))
    q, s = O.fp4_act_quant(x)
    a = O.fp4_act_dequant(q, s)
    ref = O.expert_forward_dequant(a, None, None, 0.0, dense=(w1, w2, w3), fp4_h=True)
    got = O.expert_forward(x, None, None, 0.0, dense=(w1, w2, w3), fp4_act=True)
    assert np.array_equal(got, ref)
    assert not np.array_equal(got, O.expert_forward(x, None, None, 0.0, dense=(w1, w2, w3)))
