"""The custom ops under torch.compile (AOTAutograd with the ops' fake
implementations and registered backward formulas): a model of converted
depthwise layers compiles without graph breaks into our ops and gives the
eager results, forward and backward, for fp16 and bf16."""
import pytest
import torch

import tdc_torch

pytestmark = pytest.mark.gpu


def _model(dtype):
    torch.manual_seed(0)
    m = torch.nn.Sequential(
        torch.nn.Conv2d(64, 64, 3, padding=1, groups=64),
        torch.nn.ReLU(),
        torch.nn.Conv2d(64, 64, 5, stride=2, padding=2, groups=64, bias=False),
        torch.nn.Conv2d(64, 64, 7, padding=3, groups=64),
    ).cuda().to(dtype)
    assert tdc_torch.convert_depthwise_convs(m) == 3
    return m


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_compiled_model_matches_eager(dtype):
    torch._dynamo.reset()
    eager = _model(dtype)
    compiled = torch.compile(_model(dtype), backend="aot_eager", fullgraph=True)
    x = torch.randn(2, 64, 30, 44, device="cuda", dtype=dtype).to(memory_format=torch.channels_last)
    xe, xc = x.clone().requires_grad_(), x.clone().requires_grad_()
    ye, yc = eager(xe), compiled(xc)
    assert torch.equal(ye, yc)
    g = torch.randn_like(ye)
    ye.backward(g)
    yc.backward(g)
    assert torch.equal(xe.grad, xc.grad)
    for pe, pc in zip(eager.parameters(), compiled.parameters()):
        assert torch.equal(pe.grad, pc.grad)
