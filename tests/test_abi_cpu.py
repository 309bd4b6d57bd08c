"""CPU-side checks of the C ABI and the host logic (no GPU compute)."""
import ctypes
import os
import re

import pytest
import torch
import torch.nn as nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "domino_draft.h")


@pytest.fixture(scope="module")
def lib():
    from domino_b200.build import build
    build()
    from domino_b200 import _lib
    return _lib.load()


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dd_[a-z_]+)\s*\(", text)))


def test_header_declares_the_bound_functions():
    from domino_b200 import _lib
    assert header_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), name


def test_version_and_argument_errors(lib):
    from domino_b200 import _lib
    assert b"sm_100a" in lib.dd_version()
    # argument validation happens before any CUDA call
    assert lib.dd_accept(None, None, 1, 16, None, None, None) == _lib.DD_EINVAL
    assert b"accept" in lib.dd_last_error(None)
    assert lib.dd_create(None, 0, None) == _lib.DD_EINVAL
    cfg = _lib.DDConfig(batch=64, steps=15, hidden=64, gru_hidden=64, emb_dim=64, vocab=100, prefix_tokens=1, dtype=0)
    h = ctypes.c_void_p()
    assert lib.dd_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == _lib.DD_EINVAL
    assert b"batch" in lib.dd_last_error(None)
    cfg.batch, cfg.hidden = 1, 60
    assert lib.dd_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == _lib.DD_EINVAL
    assert lib.dd_set_timing(None, 1) == _lib.DD_EINVAL
    assert lib.dd_destroy(None) == _lib.DD_OK


class _Head(nn.Module):
    def __init__(self, proj, gru=None):
        super().__init__()
        self.embed_proj = proj
        self.prefix_gru = gru or nn.GRU(8, 8, batch_first=True, bias=False)


class _Tgt(nn.Module):
    def __init__(self):
        super().__init__()
        self.model = nn.Module()
        self.model.embed_tokens = nn.Embedding(10, 8)


def _mk(proj, dtype=torch.bfloat16, gru=None, device="cuda"):
    from domino_b200 import DraftCorrectionGraphRunner
    return DraftCorrectionGraphRunner(_Head(proj, gru).to(dtype), _Tgt().to(dtype), 1, 15, 8, 8, 10, 1, device)


def test_runner_validates_like_the_reference():
    """Checks of code/kernel/domino.py:30-48, 265-270 (and the SiLU guard)."""
    with pytest.raises(TypeError):
        _mk(nn.Linear(16, 10))
    with pytest.raises(ValueError):
        _mk(nn.Sequential(nn.Linear(16, 10)))
    with pytest.raises(ValueError):
        _mk(nn.Sequential(nn.SiLU(), nn.Linear(16, 10)))
    with pytest.raises(ValueError):
        _mk(nn.Sequential(nn.Linear(15, 12), nn.SiLU(), nn.Linear(12, 10)))
    with pytest.raises(NotImplementedError):
        _mk(nn.Sequential(nn.Linear(16, 12), nn.Softplus(), nn.Linear(12, 10)))
    with pytest.raises(NotImplementedError):
        _mk(nn.Sequential(nn.Linear(16, 12), nn.SiLU(), nn.Linear(12, 10)), dtype=torch.float64)
    with pytest.raises(ValueError):
        _mk(nn.Sequential(nn.Linear(16, 12), nn.SiLU(), nn.Linear(12, 10)),
            gru=nn.GRU(8, 8, num_layers=2, batch_first=True))
    with pytest.raises(RuntimeError):
        _mk(nn.Sequential(nn.Linear(16, 12), nn.SiLU(), nn.Linear(12, 10)), device="cpu")


def test_middle_kinds_follow_the_reference_branches():
    """One SiLU (alone or the single child of a Sequential) is the reference's
    fused path (code/kernel/domino.py:280-289); everything else is its PyTorch
    branch, which the kernels implement for these activations."""
    from domino_b200 import _lib
    from domino_b200.runner import middle_kind

    assert middle_kind(nn.SiLU()) == _lib.DD_MIDDLE_SILU
    assert middle_kind(nn.Sequential(nn.SiLU())) == _lib.DD_MIDDLE_SILU
    assert middle_kind(nn.Sequential(nn.SiLU(), nn.Dropout(0.1))) == _lib.DD_MIDDLE_SILU_ROUNDED
    assert middle_kind(nn.Sequential(nn.Sequential(nn.SiLU(), nn.Dropout(0.1)))) == _lib.DD_MIDDLE_SILU_ROUNDED
    assert middle_kind(nn.Identity()) == _lib.DD_MIDDLE_IDENTITY
    assert middle_kind(nn.Sequential(nn.GELU())) == _lib.DD_MIDDLE_GELU
    assert middle_kind(nn.GELU(approximate="tanh")) == _lib.DD_MIDDLE_GELU_TANH
    assert middle_kind(nn.ReLU()) == _lib.DD_MIDDLE_RELU
    assert middle_kind(nn.Tanh()) == _lib.DD_MIDDLE_TANH
    assert middle_kind(nn.Sequential(nn.Dropout(0.0), nn.Sigmoid())) == _lib.DD_MIDDLE_SIGMOID
    for bad in (nn.Softplus(), nn.Sequential(nn.ReLU(), nn.Tanh()), nn.LeakyReLU()):
        with pytest.raises(NotImplementedError):
            middle_kind(bad)
