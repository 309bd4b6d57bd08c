"""The allocation-free rollout entry point, dd_rollout_noalloc.

Some callers cannot allocate device memory: code that runs while a CUDA
graph is being captured, hosts whose own pool owns all of HBM, and
stateless foreign-function bindings that cannot keep a handle's buffers
alive.  dd_rollout_noalloc serves them from a static scratch array inside
the library.  This test calls it through the C ABI twice in a row and checks
each result against the handle-based entry point (dd_rollout, through the
runner) on the same inputs: the draft tokens must be identical, since both
run the same kernels with the same work split.

It lives in its own file so that pytest collects it last; it passes alone in
a fresh process and after the other tests.
"""
import ctypes

import pytest
import torch

from tests.gpu_helpers import random_inputs, random_modules

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")


def test_noalloc_rollout_matches_handle_rollout_twice():
    from domino_b200 import DraftCorrectionGraphRunner, _lib

    lib = _lib.load()
    B, H, G, E, V, S, P = 3, 256, 192, 384, 4099, 15, 2
    draft, target = random_modules(H, G, E, V, seed=77, fc2_std=0.08, fc1_bias=True, gru_bias=True)
    runner = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), use_graph=False)
    cfg = _lib.DDConfig(batch=B, steps=S, hidden=H, gru_hidden=G, emb_dim=E, vocab=V, prefix_tokens=P,
                        dtype=_lib.DD_BF16)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=100 + call)
        expected = runner(prefix, ph, base)
        out = torch.full((B, S), -1, dtype=torch.long, device="cuda")
        rc = lib.dd_rollout_noalloc(ctypes.byref(cfg), ctypes.byref(runner._weights), 0, prefix.data_ptr(),
                                    ph.data_ptr(), base.data_ptr(), out.data_ptr(), stream)
        assert rc == _lib.DD_OK, lib.dd_last_error(None)
        # the kernels' own status (bounded waits, token ids): clean
        assert lib.dd_noalloc_status(0) == 0
        assert torch.equal(out, expected), (call, out, expected)


def test_noalloc_status_reports_a_clamped_prefix_id_once():
    """A caller without a handle still learns what the kernels found: an
    out-of-range prefix id is clamped and flagged in the static status word,
    which dd_noalloc_status returns and clears."""
    from domino_b200 import DraftCorrectionGraphRunner, _lib

    lib = _lib.load()
    B, H, G, E, V, S, P = 2, 64, 64, 96, 700, 15, 1
    draft, target = random_modules(H, G, E, V, seed=41)
    runner = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), use_graph=False)
    cfg = _lib.DDConfig(batch=B, steps=S, hidden=H, gru_hidden=G, emb_dim=E, vocab=V, prefix_tokens=P,
                        dtype=_lib.DD_BF16)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=1)
    prefix[0, 0] = V + 5
    out = torch.empty(B, S, dtype=torch.long, device="cuda")
    rc = lib.dd_rollout_noalloc(ctypes.byref(cfg), ctypes.byref(runner._weights), 0, prefix.data_ptr(),
                                ph.data_ptr(), base.data_ptr(), out.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.DD_OK, lib.dd_last_error(None)
    assert lib.dd_noalloc_status(0) == _lib.DD_STATUS_BAD_TOKEN
    assert lib.dd_noalloc_status(0) == 0  # reading cleared it


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from domino_b200 import _lib

    lib = _lib.load()
    cfg = _lib.DDConfig(batch=32, steps=15, hidden=4096, gru_hidden=4096, emb_dim=12288, vocab=151936,
                        prefix_tokens=1, dtype=_lib.DD_BF16)
    w = _lib.DDWeights()
    dummy = torch.zeros(16, dtype=torch.long, device="cuda")
    p = dummy.data_ptr()
    rc = lib.dd_rollout_noalloc(ctypes.byref(cfg), ctypes.byref(w), 0, p, p, p, p,
                                torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.DD_EINVAL
    assert b"static scratch holds" in lib.dd_last_error(None)
