"""CPU-side checks of the drop-in boundary: the C-ABI library loads, exports every entry
point the headers declare, and its host helpers reproduce the reference exactly."""
import os
import re

import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, TINY
from oracle import ref

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(mm_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    L = E.lib()
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n


def test_parameter_count_matches_reference_config():
    assert E.parameter_count(MLA36M) == 35763840 == MLA36M.parameter_count()
    assert E.parameter_count(TINY) == 26704 == TINY.parameter_count()


@pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("seed", [0, 1, 12345])
def test_init_params_bit_exact_with_reference(seed):
    assert np.array_equal(E.init_params(TINY, seed), ref.Session(TINY, seed).params())


@pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built")
def test_cosine_schedule_matches_reference():
    for done in range(0, 130, 3):
        for warm in (0, 10):
            assert E.cosine_learning_rate(done, 100, warm, 1e-3, 0.1) == \
                ref.cosine_lr(done, 100, warm, 1e-3, 0.1)


def test_context_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(E.EngineError) as e:
        E.CudaExecution(TINY)
    assert e.value.name == "gpu_error"
