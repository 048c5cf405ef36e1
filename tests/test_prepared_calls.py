"""The prepared calls (ops.LayerStep, ops.W8Linear, ops.W8A8Linear) on CPU: they check their weights once, at
construction, and refuse CPU tensors there (the ops have no CPU path); nothing here launches a kernel."""
import pytest
import torch

from qwenfast_b200 import ops
from qwenfast_b200.ops import LayerStep, MoELayerWeights, W8A8Linear, W8Linear

BF = torch.bfloat16


def test_w8_prepared_calls_refuse_cpu_weights():
    q = torch.zeros(256, 256, dtype=torch.int8)
    with pytest.raises(RuntimeError, match="W8Linear: q and s must be CUDA tensors"):
        W8Linear(q, torch.zeros(256, 2, dtype=BF))
    with pytest.raises(RuntimeError, match="W8A8Linear: q and sw must be CUDA tensors"):
        W8A8Linear(q, torch.zeros(256, dtype=torch.float32))


def test_layer_step_refuses_cpu_weights():
    H, E, I = 256, 16, 128
    lw = MoELayerWeights(torch.zeros(E, H, dtype=BF), torch.zeros(E, 2 * I * H // 8, dtype=torch.int32),
                         torch.zeros(E, 2 * I * H // 128, dtype=BF), torch.zeros(E, H * I // 8, dtype=torch.int32),
                         torch.zeros(E, H * I // 128, dtype=BF), None, None, None, H, I, E, 0)
    with pytest.raises(RuntimeError, match="LayerStep: the weights must be CUDA tensors"):
        LayerStep(lw, 4, {})


def test_prepared_calls_are_exported():
    import qwenfast_b200
    for name in ("LayerStep", "W8Linear", "W8A8Linear"):
        assert name in qwenfast_b200.__all__ and getattr(qwenfast_b200, name) is getattr(ops, name)
