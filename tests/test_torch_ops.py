"""The TORCH_LIBRARY(dsv4moe) op layer on the CPU: the library loads, every
op has the expected schema, the fake kernels give the right output shapes on
meta tensors (so the ops trace without a GPU), and the host op ``read_into``
behaves as the reference loader (native_packed_loader.cpp:26-68)."""

import os
import tempfile

import pytest
import torch

OPS = ["moe_forward", "moe_forward_out", "moe_workspace_bytes", "expert_forward", "gate_route", "gate_logits",
       "gate_topk", "act_quant", "materialize", "build_scale_atoms", "build_shared_scale_atoms", "ep_dispatch",
       "ep_expert_forward", "ep_combine", "ep_dispatch_p2p", "ep_expert_forward_p2p", "ep_combine_p2p",
       "read_into", "sparse_attn", "build_fp8_weight_atoms", "fp8_linear", "fp4_act_quant"]


@pytest.fixture(scope="module")
def dsv4():
    from spark_b200 import ops

    return ops.load()


def test_every_op_is_registered(dsv4):
    for name in OPS:
        op = getattr(dsv4, name)
        assert op.default._schema.name == f"dsv4moe::{name}"
    assert "Tensor?[] layer, int[] dims, float[] scalars" in str(dsv4.moe_forward.default._schema)


def test_fake_kernels_give_output_shapes_on_meta(dsv4):
    from spark_b200 import ops

    H, I, E, k, T = 1024, 512, 16, 4, 7
    m = torch.device("meta")
    x = torch.empty(T, H, dtype=torch.bfloat16, device=m)
    layer = [torch.empty(E, H, dtype=torch.float32, device=m), torch.empty(E, device=m),
             torch.empty(E * 4096, dtype=torch.uint8, device=m), torch.empty(E * 512, dtype=torch.uint8, device=m),
             torch.empty(E, dtype=torch.int32, device=m)] + [None] * 4
    dims = [H, I, E, k, 0, E, 4096, 512]
    y = dsv4.moe_forward(x, layer, dims, [2.5, 10.0])
    assert y.shape == (T, H) and y.dtype == torch.bfloat16 and y.device == m
    w, idx, logits = dsv4.gate_route(x, layer[0], layer[1], k, 2.5)
    assert w.shape == (T, k) and idx.dtype == torch.int64 and logits.shape == (T, E)
    q, s = dsv4.act_quant(x)
    assert q.shape == (T, H) and s.shape == (T, H // 128) and q.dtype == torch.uint8
    q4, s4 = dsv4.fp4_act_quant(x)
    assert q4.shape == (T, H // 2) and s4.shape == (T, H // 32) and q4.dtype == torch.uint8
    assert dsv4.gate_logits(x, layer[0]).shape == (T, E)
    assert dsv4.expert_forward(x, 0, None, layer, dims, [1.0, 0.0]).shape == (T, H)
    assert ops.OPS_LIB.name == "libdsv4moe_torch.so"
    q = torch.empty(2, 3, 64, 512, dtype=torch.bfloat16, device=m)
    kv = torch.empty(2, 100, 512, dtype=torch.bfloat16, device=m)
    o = dsv4.sparse_attn(q, kv, torch.empty(64, device=m), torch.empty(2, 3, 16, dtype=torch.int32, device=m), 0.04)
    assert o.shape == q.shape and o.dtype == torch.bfloat16
    atoms = dsv4.build_fp8_weight_atoms(torch.empty(4, 8, dtype=torch.uint8, device=m), 512, 1024)
    assert atoms.dtype == torch.uint8 and atoms.numel() > 0
    y = dsv4.fp8_linear(torch.empty(2, 5, 1024, dtype=torch.bfloat16, device=m),
                        torch.empty(512, 1024, dtype=torch.uint8, device=m), atoms)
    assert y.shape == (2, 5, 512) and y.dtype == torch.bfloat16


def test_read_into_op_matches_the_reference_loader():
    from spark_b200 import ops

    dsv4 = ops.load()
    data = bytes(range(256)) * 8
    with tempfile.NamedTemporaryFile() as f:
        f.write(data)
        f.flush()
        fd = os.open(f.name, os.O_RDONLY)
        try:
            dst = torch.zeros(4096, dtype=torch.uint8)
            assert dsv4.read_into(fd, dst, 100, 10) == 100
            assert bytes(dst[:100].tolist()) == data[10:110]
            assert dsv4.read_into(fd, dst, 2000, 1000) == 1048  # short count at EOF
            with pytest.raises(RuntimeError, match="offset must be non-negative"):
                dsv4.read_into(fd, dst, 10, -1)
            with pytest.raises(RuntimeError, match="destination tensor is too small"):
                dsv4.read_into(fd, torch.zeros(4, dtype=torch.uint8), 10, 0)
        finally:
            os.close(fd)
    with pytest.raises(RuntimeError, match="pread failed: Bad file descriptor"):
        dsv4.read_into(987654, torch.zeros(16, dtype=torch.uint8), 8, 0)
