"""vLLM plugin that applies FOLD to the drafter (fold/vllm_plugin.py of the reference).

vLLM loads general plugins in every process. When FOLD_CONFIG is set (a JSON object with the
keyword arguments of fold_b200.attention.install), the GPU model runner is wrapped so that the
drafter gets full KV storage when it is loaded and FOLD is installed right before CUDA graph
capture. Entry point: vllm.general_plugins: fold = fold_b200.vllm_plugin:register.

    FOLD_CONFIG='{"window": 2048, "alpha": 2.0}'
"""
import json
import logging
import os

import torch

logger = logging.getLogger("vllm.fold")


def register():
    raw = os.environ.get("FOLD_CONFIG")
    if not raw:
        return
    config = json.loads(raw)
    from vllm.v1.worker.gpu.model_runner import GPUModelRunner

    if getattr(GPUModelRunner, "_fold", False):
        return
    from .attention import install, use_full_draft_storage

    original_load, original_capture = GPUModelRunner.load_model, GPUModelRunner.capture_model

    def load_model(self, *args, **kwargs):
        original_load(self, *args, **kwargs)
        if getattr(self.speculator, "model", None) is not None:
            use_full_draft_storage(self.speculator)

    def capture_model(self, *args, **kwargs):
        if getattr(self.speculator, "model", None) is not None:
            with torch.inference_mode():
                report = install(self.speculator, **config)
            logger.info("FOLD installed: %s", report)
        return original_capture(self, *args, **kwargs)

    GPUModelRunner.load_model = load_model
    GPUModelRunner.capture_model = capture_model
    GPUModelRunner._fold = True
