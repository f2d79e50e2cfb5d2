"""The token-loop tests' synthetic model and plan structures (the package's
qwen_b200.plans, which the benchmark uses too)."""
from qwen_b200.plans import (CALLBACK, FFN, FULL_LAYERS, HEAD_DIM, HEADS, HIDDEN, LAYERS, V, VOCAB,  # noqa: F401
                             Linear, LinearLayerPlanC, Mlp, MlpPlanC, TokenModel, attention_stand_in, bfp8_matrix)
