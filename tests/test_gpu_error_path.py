"""The device-side error path on one GPU: a pipeline wait that runs out ends the kernel through
its bounded-wait exit and the call returns RV_E_DEVICE, and the next call on the same context is
parity-green (the reference's contract: errors propagate, never silent defaults,
crates/ripvec-core/src/backend/mod.rs:53-54).

The failure is made by the library's test hook rv_debug_stall_attention: the first tile's score
signal of every persistent attention CTA is withheld and the waits are bounded by about a
millisecond of SM cycles.  Nothing faults, traps or spins without bound; the host reads the
error word after the launch."""

import numpy as np
import pytest

from helpers import TINY_MODERN, modern_cfg, row_cosines
from oracle import modern_bert
from ripvec_b200 import EmbedBackend, synth
from ripvec_b200 import _lib as L
from ripvec_b200._lib import RvError
from test_gpu_kernels import _attention_ref, _stream, _torch

pytestmark = pytest.mark.gpu
LIMIT = 2_000_000  # SM cycles (about a millisecond)


@pytest.fixture
def stall():
    lib = L.lib()
    yield lib
    assert lib.rv_debug_stall_attention(0, 0) == L.RV_OK


def test_attention_wait_timeout_returns_device_error_then_recovers(cuda_device, stall, monkeypatch):
    torch = _torch()
    monkeypatch.setenv("RV_ATTN_TC", "1")
    heads, hd = 12, 64
    lengths = [300, 17, 512, 129]
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    T = int(cu[-1])
    rng = np.random.default_rng(5)
    qkv = torch.from_numpy(rng.standard_normal((T, 3 * heads * hd)).astype(np.float32)).to(torch.bfloat16).cuda()
    ctx = torch.zeros(T, heads * hd, device="cuda", dtype=torch.bfloat16)

    def run():
        return stall.rv_op_attention(L.RV_DTYPE_BF16, qkv.data_ptr(), ctx.data_ptr(), cu.ctypes.data, len(lengths),
                                     heads, hd, -1, float(1.0 / np.sqrt(hd)), _stream())

    assert stall.rv_debug_stall_attention(1, 0) == L.RV_E_INVALID  # a limit is required
    assert stall.rv_debug_stall_attention(1, LIMIT) == L.RV_OK
    assert run() == L.RV_E_DEVICE
    assert run() == L.RV_E_DEVICE  # the error word was cleared and is raised again
    assert stall.rv_debug_stall_attention(0, 0) == L.RV_OK
    assert run() == L.RV_OK
    ref = _attention_ref(qkv.float().cpu().numpy(), cu, heads, hd, -1)
    assert np.abs(ctx.float().cpu().numpy() - ref).max() < 3e-2


def test_model_call_reports_the_timeout_and_the_context_stays_usable(cuda_device, stall):
    w = synth.random_weights(TINY_MODERN, seed=3, qk_std=0.2)
    ids, cu = synth.packed_ids(np.array([200, 64, 700, 5], np.int32), TINY_MODERN.vocab, seed=4)
    ref = modern_bert.embed_batch(w, modern_cfg(TINY_MODERN), ids, cu)
    be = EmbedBackend(TINY_MODERN, w, dtype="bf16")
    before = be.embed_packed(ids, cu)
    assert stall.rv_debug_stall_attention(1, LIMIT) == L.RV_OK
    with pytest.raises(RvError) as e:
        be.embed_packed(ids, cu)
    assert e.value.code == L.RV_E_DEVICE
    assert "pipeline wait expired" in str(e.value)
    assert stall.rv_debug_stall_attention(0, 0) == L.RV_OK
    after = be.embed_packed(ids, cu)
    np.testing.assert_array_equal(after, before)
    assert row_cosines(after, ref).min() >= 0.999
    be.close()
