"""CPU checks of the oracle's number formats and routing arithmetic."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O


def test_e4m3_table_matches_torch():
    codes = torch.arange(256, dtype=torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).float().numpy()
    ours = O.E4M3_VALUES
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(ours))
    assert np.array_equal(ref[~nan], ours[~nan])


def test_e4m3_rounding_matches_torch():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 50,
        rng.standard_normal(50000).astype(np.float32) * 1e-2,   # subnormal range
        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11], np.float32),
    ])
    x = np.clip(x, -448, 448)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    ours = O.f32_to_e4m3_codes(x)
    # torch keeps the sign of zero the same way
    assert np.array_equal(ref, ours)


def test_e4m3_saturates():
    assert O.f32_to_e4m3_codes(np.array([460.0, -1e6], np.float32)).tolist() == [0x7E, 0xFE]


def test_e2m1_values_follow_ocp_formula():
    for c in range(16):
        s = -1.0 if c & 8 else 1.0
        e, m = (c >> 1) & 3, c & 1
        v = s * (0.5 * m if e == 0 else 2.0 ** (e - 1) * (1 + 0.5 * m))
        assert O.E2M1_VALUES[c] == np.float32(v)


def test_unpack_low_nibble_first():
    packed = np.array([[0x21, 0x7F]], np.uint8)
    assert O.unpack_e2m1(packed).tolist() == [[0.5, 1.0, -6.0, 6.0]]


def test_e8m0_matches_torch():
    codes = torch.arange(0, 255, dtype=torch.uint8)
    ref = codes.view(torch.float8_e8m0fnu).float().numpy()
    assert np.array_equal(ref, O.e8m0_to_f32(codes.numpy()))


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(100000) * 1e3).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(ref, O.round_bf16(x))


def test_act_quant_properties():
    rng = np.random.default_rng(3)
    x = O.round_bf16(rng.standard_normal((16, 512)).astype(np.float32))
    x[0, :128] = 0.0                       # amax clamped at 1e-4
    x[1, :128] = 0.0
    x[1, 5] = 3.5                          # amax = 1.75 * 2^1: scale exactly 2^-7
    q, s = O.act_quant(x)
    assert q.shape == x.shape and s.shape == (16, 4)
    assert s[1, 0] == 127 - 7
    deq = O.act_dequant(q, s)
    # round-to-nearest in e4m3: half an ulp = 2^-4 of the value in the normal
    # range, half the subnormal quantum (2^-10 of the scale) below it
    scale = np.repeat(O.e8m0_to_f32(s), 128, 1)
    assert np.all(np.abs(deq - x) <= np.maximum(np.abs(x) * 2.0 ** -4, scale * 2.0 ** -10))
    assert deq[1, 5] == 3.5 and O.decode_e4m3(q[1, 5]) == 448
    assert np.all(np.abs(O.decode_e4m3(q)) <= 448)


def test_sigmoid_canonical_accuracy():
    x = np.linspace(-30, 30, 200001).astype(np.float32)
    ref = 1.0 / (1.0 + np.exp(-x.astype(np.float64)))
    got = O.sigmoid_canonical(x).astype(np.float64)
    assert np.max(np.abs(got - ref) / ref) < 5e-7


def test_route_from_logits_matches_torch_topk():
    rng = np.random.default_rng(4)
    logits = rng.standard_normal((64, 256)).astype(np.float32)
    bias = (rng.random(256).astype(np.float32) - 0.5) * 0.2
    w, idx = O.route_from_logits(logits, bias, 6, 2.5)
    s = torch.from_numpy(O.sigmoid_canonical(logits))
    ti = torch.topk(s + torch.from_numpy(bias), 6, dim=-1).indices
    assert np.array_equal(ti.numpy(), idx)
    tw = s.gather(1, ti)
    tw = tw / tw.sum(-1, keepdim=True) * 2.5
    np.testing.assert_allclose(tw.numpy(), w, rtol=5e-7, atol=0)  # torch sums in another order


def test_route_ties_pick_lower_id():
    logits = np.zeros((1, 16), np.float32)
    w, idx = O.route_from_logits(logits, None, 4, 1.0)
    assert idx.tolist() == [[0, 1, 2, 3]]
    assert np.allclose(w, 0.25)


def test_sf_atoms_layout():
    s = np.arange(256 * 8, dtype=np.int64).reshape(256, 8) % 251
    s = s.astype(np.uint8)
    at = O.sf_atoms(s).reshape(2, 2, 32, 4, 4)  # nb, kt, m0, m1, b
    for nb in range(2):
        for kt in range(2):
            for m0 in range(32):
                for m1 in range(4):
                    assert np.array_equal(at[nb, kt, m0, m1], s[nb * 128 + m1 * 32 + m0, kt * 4:(kt + 1) * 4])


@pytest.mark.parametrize("limit", [0.0, 10.0])
def test_expert_forward_linear_in_route_weight(limit):
    rng = np.random.default_rng(5)
    H, I = 256, 128
    blk = np.concatenate([rng.integers(119, 124, 3 * I * H // 32), rng.integers(0, 256, 3 * I * H // 2)])
    ew = O.expert_from_block(blk.astype(np.uint8), H, I)
    x = O.round_bf16(rng.standard_normal((3, H)).astype(np.float32))
    y1 = O.expert_forward(x, ew, np.ones(3, np.float32), limit)
    y0 = O.expert_forward(x, ew, None, limit)
    assert np.array_equal(y0, y1)


def test_route_plan_follows_torch_where_order():
    """Segment e lists torch.where(indices == e)'s tokens in order; padding to
    32 rows; the shared segment is the identity; tiles cover each segment."""
    g = torch.Generator().manual_seed(5)
    T, k, E, bn = 77, 4, 16, 32
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    p = O.route_plan(idx.numpy(), E, bn, T)
    for e in range(E):
        rows, top = torch.where(idx == e)
        s0, c = int(p["seg_start"][e]), int(p["counts"][e])
        assert np.array_equal(p["slot_token"][s0:s0 + c], rows.numpy())
        assert np.array_equal(p["route_slot"][(rows * k + top).numpy()], np.arange(s0, s0 + c))
        assert (p["slot_token"][s0 + c:int(p["seg_start"][e + 1])] == -1).all()
        assert int(p["seg_start"][e + 1]) - s0 == -(-c // 32) * 32
    s0 = int(p["seg_start"][E])
    assert np.array_equal(p["slot_token"][s0:s0 + T], np.arange(T))
    assert sum(t[2] for t in p["tiles"]) == T * k + T


def test_hash_route_uses_the_table_and_renormalises():
    rng = np.random.default_rng(3)
    T, E, k, vocab = 9, 16, 4, 50
    logits = rng.standard_normal((T, E)).astype(np.float32)
    table = np.stack([rng.permutation(E)[:k] for _ in range(vocab)])
    ids = rng.integers(0, vocab, T)
    w, idx = O.hash_route(logits, table, ids, 2.5)
    assert np.array_equal(idx, table[ids])
    assert np.allclose(w.sum(1), 2.5, rtol=1e-6)
    s = O.sigmoid_canonical(logits)
    assert np.allclose(w / 2.5, s[np.arange(T)[:, None], idx] / s[np.arange(T)[:, None], idx].sum(1, keepdims=True),
                       rtol=1e-6)
