"""GPT / rGPT modules with the reference's Python API (model/__init__.py of the reference)."""
from .attention import Attention
from .feed_forward import FeedForward
from .gpt import GPT
from .kernels import FusedLinearActivationFunction
from .norm import (AsymmetricHyperballNorm, DualElasticBallNorm, ElasticBallNorm, HybridElasticNorm, HyperballNorm,
                   L2Norm, QKNorm, RMSNorm, functional_l2_norm, functional_rms_norm, get_norm_fn)
from .rope import RotaryEmbedding
from .transformer_block import TransformerBlock

__all__ = [
    "Attention", "FeedForward", "GPT", "QKNorm", "TransformerBlock", "FusedLinearActivationFunction",
    "RMSNorm", "L2Norm", "HybridElasticNorm", "ElasticBallNorm", "DualElasticBallNorm", "AsymmetricHyperballNorm",
    "HyperballNorm", "functional_rms_norm", "functional_l2_norm", "get_norm_fn", "RotaryEmbedding",
]
