"""Host side of the fused row-parallel linear in the vLLM plugin (no GPU): when it is switched
on, which linears it takes, and that a routed linear returns the op's result in vLLM's
(output, bias) form while inputs it cannot take go to vLLM's own forward."""
import sys
import types
from unittest import mock

import torch
import torch.nn as nn

from test_vllm_tp import vllm_faked


class _RowLinear(nn.Module):
    """The attributes of vLLM's RowParallelLinear that the plugin reads."""

    def __init__(self, n_out=16, k=32, dtype=torch.bfloat16, bias=False):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(n_out, k).to(dtype), requires_grad=False)
        self.bias = nn.Parameter(torch.zeros(n_out)) if bias else None
        self.input_is_parallel, self.reduce_results, self.return_bias = True, True, True

    def forward(self, x):
        return x.float() @ self.weight.float().t() * 0, None  # "vLLM's path": zeros, so a routed call shows


class _Twice:
    """Stands in for TPRowLinear: records its calls and returns 2 x . W^T."""

    def __init__(self):
        self.calls = 0

    def __call__(self, x, w):
        self.calls += 1
        return 2 * (x.float() @ w.float().t()).to(x.dtype)


def _config(extra=None, eager=True):
    return types.SimpleNamespace(additional_config=extra or {},
                                 model_config=types.SimpleNamespace(enforce_eager=eager),
                                 scheduler_config=types.SimpleNamespace(max_num_batched_tokens=8))


def test_switch_and_routing():
    with vllm_faked():
        sys.modules.pop("micro_engram_vllm.model", None)
        from micro_engram_vllm import model as M
        from micro_engram_fork_b200.ops.registry import add_tp_linear

        assert not M.fused_tp_wanted(_config(), environ={})
        assert M.fused_tp_wanted(_config(), environ={"MICRO_ENGRAM_FUSED_TP": "1"})
        assert not M.fused_tp_wanted(_config({"micro_engram_fused_tp": False}), environ={"MICRO_ENGRAM_FUSED_TP": "1"})
        assert M.fused_tp_wanted(_config({"micro_engram_fused_tp": True}), environ={})

        assert M._fusable(_RowLinear())
        assert not M._fusable(_RowLinear(dtype=torch.float32))
        assert not M._fusable(_RowLinear(bias=True))
        assert not M._fusable(_RowLinear(n_out=12))

        lin, op = _RowLinear(), _Twice()
        M._route_row_parallel(lin, add_tp_linear(op), rows=8)
        x = torch.randn(5, 32).to(torch.bfloat16)
        y, b = lin(x)
        assert b is None and op.calls == 1
        assert torch.equal(y, 2 * (x.float() @ lin.weight.float().t()).to(torch.bfloat16))
        assert lin(torch.randn(9, 32).to(torch.bfloat16))[0].abs().sum() == 0  # more rows than built for
        assert lin(torch.randn(5, 32))[0].abs().sum() == 0  # not bf16
        assert op.calls == 1

        # TP = 1 (the fake's world without a process group) or no eager: nothing is routed
        model = types.SimpleNamespace(model=types.SimpleNamespace(layers=[]))
        assert M.fuse_row_parallel(model, _config({"micro_engram_fused_tp": True})) == 0
        with mock.patch.object(M, "get_tensor_model_parallel_world_size", lambda: 2):
            assert M.fuse_row_parallel(model, _config({"micro_engram_fused_tp": True}, eager=False)) == 0
    sys.modules.pop("micro_engram_vllm.model", None)
