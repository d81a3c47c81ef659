"""B200-native (sm_100a) backend for Parrot XL's MoE block, RMSNorm and Block AttnRes.

Drop-in for the reference ``parrot`` package's inference API:

    from parrot_b200 import ModelConfig, Parrot
    model = Parrot(ModelConfig()).to("cuda", torch.bfloat16).eval()
    with torch.inference_mode():
        out = model(ids.cuda())

The hot path runs in ``libparrot_b200.so`` (C ABI: ``include/parrot_b200.h``);
``parrot_b200.bridge`` holds the module-level functions a patched reference
``parrot/model.py`` calls for ``moe_backend="b200"`` / ``depth_backend="b200"``.
"""
from .model import (Block, DepthMix, GenerationState, GlobalMLA, LocalGQA, LocalKVCache,
                    MLALatentCache, ModelConfig, ModelOutput, MoE, Parrot, RMSNorm, SwiGLU)

__all__ = ["Block", "DepthMix", "GenerationState", "GlobalMLA", "LocalGQA", "LocalKVCache",
           "MLALatentCache", "ModelConfig", "ModelOutput", "MoE", "Parrot", "RMSNorm", "SwiGLU"]
