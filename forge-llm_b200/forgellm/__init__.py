"""forgellm -- forge-llm's training hot path on B200 (sm_100a).

The same operator API as forge-llm's src/L2/tensor.js, src/L2/autograd.js and
src/L6/train.js (and, in `infer`, the decode side: src/L4/nn.js QuantLinear,
src/L5/attention.js, src/L6/transformer.js), computed by the hand-written CUDA
kernels of libforgecu.so
(C-ABI: include/forgecu.h).  There is no CPU fallback: without the library or
a CUDA device every operator raises ``ForgeCUError``.
"""
from ._lib import ForgeCUError, PRECISIONS
from .autograd import (Adam, Node, backward, gradCheck, leaf, linear, noGrad, op, param,
                       resetTape, softmaxCE, tape)
from .tensor import (causalAttn, causalAttnBatch, crossEntropyMean, embedLookup, matmulT,
                     ropeRows, rmsNorm, sliceCols, swigluRows, weightedSum)
from .train import RNG, Config, TrainableTransformer, initWeights, train
from .checkpoint import load_checkpoint, save_checkpoint
from .infer import (KVCache, PagedKVCache, QuantLinear, Transformer, attentionDecode, attentionNaive,
                    flashAttention)


def set_precision(mode: str) -> None:
    """Arithmetic of the contractions on the current device: "fp32"
    (CUDA cores, parity), "fp32tc" (parity, matmulT on the tcgen05 tensor
    cores through a three-way bf16 split) or "bf16" (tcgen05 tensor cores)."""
    from .autograd import ctx
    ctx().set_precision(PRECISIONS[mode])


__all__ = [
    "ForgeCUError", "Adam", "Node", "backward", "gradCheck", "leaf", "linear", "noGrad", "op",
    "param", "resetTape", "softmaxCE", "tape", "causalAttn", "causalAttnBatch",
    "crossEntropyMean", "embedLookup", "matmulT", "ropeRows", "rmsNorm", "sliceCols",
    "swigluRows", "weightedSum", "RNG", "Config", "TrainableTransformer", "initWeights", "train",
    "set_precision", "QuantLinear", "KVCache", "PagedKVCache", "Transformer", "attentionDecode",
    "attentionNaive", "flashAttention",
]
