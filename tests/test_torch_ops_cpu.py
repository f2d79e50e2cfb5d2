"""The PyTorch operator library (torch.ops.qwen_b200, csrc/torch_ops.cpp)
without a GPU: it loads, registers every operator of the device-level API
with its schema, and has no CPU kernel -- a CPU tensor raises instead of
falling back to anything."""
import pytest
import torch

OPS = {
    "quant_block64": "quant_block64(Tensor x) -> (Tensor, Tensor)",
    "bfp8_gemv": "bfp8_gemv(Tensor x, Tensor mant, Tensor exps, str mode=\"exact\") -> Tensor",
    "bfp8_gemv_q": "bfp8_gemv_q(Tensor xq, Tensor xs, Tensor mant, Tensor exps, str mode=\"exact\") -> Tensor",
    "lm_head_bf16": "lm_head_bf16(Tensor h, Tensor E, int k) -> (Tensor, Tensor, Tensor, Tensor)",
    "lm_head_bfp8": "lm_head_bfp8(Tensor h, Tensor mant, Tensor exps, int k) -> (Tensor, Tensor, Tensor, Tensor)",
    "quant_planes": "quant_planes(Tensor x) -> (Tensor, Tensor)",
    "bfp8_gemm_tc": "bfp8_gemm_tc(Tensor planes, Tensor xs_t, Tensor mant, Tensor exps) -> Tensor",
    "sample_topk": "sample_topk(Tensor ids, Tensor scores, Tensor n, float temperature, int top_k, float top_p, "
                   "Tensor(a!) rng_state) -> Tensor",
    "pack_bfp8": "pack_bfp8(Tensor w) -> (Tensor, Tensor)",
}


def test_operator_library_registers_every_op():
    from qwen_b200 import _lib

    T = _lib.torch_ops()
    for name, schema in OPS.items():
        assert str(getattr(T, name).default._schema) == "qwen_b200::" + schema, name


def test_operators_have_no_cpu_fallback():
    from qwen_b200 import _lib

    T = _lib.torch_ops()
    with pytest.raises(NotImplementedError):
        T.bfp8_gemv(torch.zeros(64), torch.zeros(1, 64, dtype=torch.int8), torch.zeros(1, 1, dtype=torch.uint8),
                    "exact")
    with pytest.raises(NotImplementedError):
        T.quant_block64(torch.zeros(64))
