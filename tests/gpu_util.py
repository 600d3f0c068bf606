"""Shared helpers of the GPU parity tests."""
import json
import os

import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import ModelConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def require_gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def golden_model(golden):
    cfg = ModelConfig.from_json(json.loads(str(golden["config"])))
    names = list(golden["param_names"])
    W = np.concatenate([golden["t:" + n + ".weight"].ravel() for n in names]).astype(np.float32)
    return cfg, names, W


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
