"""The drop-in modules construct on the CPU with the official names, shapes
and dtypes (no kernels run)."""

import torch

from spark_b200.moe import FP4, E4M3, E8M0, Expert, ExpertArena, ModelArgs, packed_block_bytes, packed_block_layout


def test_packed_block_layout_matches_manifest_sizes():
    lay = packed_block_layout(4096, 2048)
    # weight-manifest.csv:4731-4733,5510-5512: 262,144-byte scales, 4,194,304-byte weights
    assert [lay[n][1] for n in ("w1.scale", "w2.scale", "w3.scale")] == [262144] * 3
    assert [lay[n][1] for n in ("w1.weight", "w2.weight", "w3.weight")] == [4194304] * 3
    assert packed_block_bytes(4096, 2048) == 13369344
    assert [lay[n][0] for n in ("w1.scale", "w2.scale", "w3.scale", "w1.weight")] == [0, 262144, 524288, 786432]


def test_routed_expert_parameters_are_views_of_one_block():
    e = Expert(1024, 512, dtype=FP4, swiglu_limit=10.0, device="cpu")
    names = dict(e.named_parameters())
    assert set(names) == {"w1.weight", "w1.scale", "w2.weight", "w2.scale", "w3.weight", "w3.scale"}
    assert e.w1.weight.dtype == FP4 and tuple(e.w1.weight.shape) == (512, 512)
    assert e.w2.scale.dtype == E8M0 and tuple(e.w2.scale.shape) == (1024, 16)
    base = e.block.data_ptr()
    lay = packed_block_layout(1024, 512)
    for n, (off, _, _, _) in lay.items():
        mod, attr = n.split(".")
        assert getattr(getattr(e, mod), attr).data_ptr() == base + off


def test_shared_expert_is_fp8():
    e = Expert(1024, 512, swiglu_limit=10.0, device="cpu")
    assert e.w1.weight.dtype == E4M3 and tuple(e.w1.weight.shape) == (512, 1024)
    assert e.w1.scale.dtype == E8M0 and tuple(e.w1.scale.shape) == (4, 8)
    assert tuple(e.w2.weight.shape) == (1024, 512) and tuple(e.w2.scale.shape) == (8, 4)


def test_arena_acquire_release_contract():
    arena = ExpertArena(2, 256, 128, device="cpu")
    a, reused_a = arena.acquire(lambda: "factory")
    b, reused_b = arena.acquire(lambda: "factory")
    assert not reused_a and not reused_b and a is not b
    c, reused_c = arena.acquire(lambda: "factory")
    assert c == "factory" and reused_c is False      # pool exhausted -> factory
    assert arena.release(a) is True
    assert arena.release(a) is False                 # already pooled
    d, reused_d = arena.acquire(lambda: "factory")
    assert d is a and reused_d is True
    off = a.w1.weight.data_ptr() - arena.buffer.data_ptr()
    assert off % arena.slot_stride == packed_block_layout(256, 128)["w1.weight"][0]
    disabled = ExpertArena(0, 256, 128, device="cpu")
    x, r = disabled.acquire(lambda: "made")
    assert x == "made" and r is False and disabled.release(x) is False


def test_model_args_defaults_are_v4_flash_shapes():
    a = ModelArgs()
    assert (a.dim, a.moe_inter_dim, a.n_routed_experts, a.n_activated_experts, a.n_shared_experts) == (
        4096, 2048, 256, 6, 1)
    assert torch.float4_e2m1fn_x2 == FP4


def test_hash_layer_gate_has_the_checkpoint_tensors():
    """Layers below n_hash_layers hold gate.tid2eid [vocab, k] int64 and no
    correction bias (weight-manifest.csv:3 vs :4724); later layers the bias."""
    from spark_b200.moe import Gate

    args = ModelArgs(dim=256, n_routed_experts=16, n_activated_experts=4, n_hash_layers=3, vocab_size=100)
    g0 = Gate(0, args, device="cpu")
    assert g0.hashed and tuple(g0.tid2eid.shape) == (100, 4) and g0.tid2eid.dtype == torch.int64
    assert set(g0.state_dict()) == {"weight", "tid2eid"}
    g3 = Gate(3, args, device="cpu")
    assert not g3.hashed and set(g3.state_dict()) == {"weight", "bias"}
