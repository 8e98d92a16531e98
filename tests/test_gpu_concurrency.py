"""Two handles driven from two host threads at once on one device, the way the MCP server calls
``embed_batch`` for queries from ``spawn_blocking`` threads while indexing runs
(ripvec-mcp/src/tools.rs:362-371, server.rs:398-429).  ctypes releases the GIL around each
library call, so the calls overlap; each thread's results must equal a single-threaded run.
The per-device one-time set-up (kernel attributes, cached SM count) is what these runs race on.
"""

import threading

import numpy as np
import pytest

from helpers import TINY_MODERN
from ripvec_b200 import EmbedBackend, synth
from ripvec_b200.index import SearchIndex

pytestmark = pytest.mark.gpu


def _run_threads(fns):
    errors = []

    def wrap(fn):
        try:
            fn()
        except BaseException as e:  # noqa: BLE001 - surfaced below
            errors.append(e)

    ts = [threading.Thread(target=wrap, args=(f,)) for f in fns]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in ts), "a thread did not finish"
    if errors:
        raise errors[0]


def test_two_encoder_contexts_from_two_threads(cuda_device):
    w = synth.random_weights(TINY_MODERN, seed=5, qk_std=0.2)
    batches = []
    for s in range(2):
        lengths = synth.uniform_lengths(40, 16, 700, seed=60 + s)
        batches.append(synth.packed_ids(lengths, TINY_MODERN.vocab, seed=70 + s))
    # single-threaded expectations, each on a fresh context
    expect = []
    for ids, cu in batches:
        be = EmbedBackend(TINY_MODERN, w, dtype="bf16", device=cuda_device)
        expect.append(be.embed_packed(ids, cu))
        be.close()
    ctxs = [EmbedBackend(TINY_MODERN, w, dtype="bf16", device=cuda_device) for _ in range(2)]
    outs = [[], []]

    def worker(i):
        ids, cu = batches[i]
        for _ in range(6):
            outs[i].append(ctxs[i].embed_packed(ids, cu))

    _run_threads([lambda: worker(0), lambda: worker(1)])
    for i in range(2):
        for o in outs[i]:
            np.testing.assert_array_equal(o, expect[i])
        ctxs[i].close()


def test_one_context_shared_by_two_threads(cuda_device):
    """Calls on one handle are serialised inside the library: two threads sharing a context get
    the same results as one."""
    w = synth.random_weights(TINY_MODERN, seed=6)
    be = EmbedBackend(TINY_MODERN, w, dtype="f16", device=cuda_device)
    data = [synth.packed_ids(synth.uniform_lengths(25, 8, 300, seed=80 + s), TINY_MODERN.vocab, seed=90 + s)
            for s in range(2)]
    expect = [be.embed_packed(ids, cu) for ids, cu in data]
    outs = [[], []]

    def worker(i):
        for _ in range(8):
            outs[i].append(be.embed_packed(*data[i]))

    _run_threads([lambda: worker(0), lambda: worker(1)])
    for i in range(2):
        for o in outs[i]:
            np.testing.assert_array_equal(o, expect[i])
    be.close()


def test_two_indexes_from_two_threads(cuda_device):
    dim = 256
    dbs = [synth.normalized_gaussian(150_000, dim, seed=100 + s) for s in range(2)]
    qs = [synth.normalized_gaussian(9, dim, seed=110 + s) for s in range(2)]
    expect = []
    for db, q in zip(dbs, qs):
        ix = SearchIndex(db, device=cuda_device)
        expect.append(ix.topk(q, 40, with_f64=True))
        ix.close()
    idxs = [SearchIndex(db, device=cuda_device) for db in dbs]
    outs = [[], []]

    def worker(i):
        for _ in range(6):
            outs[i].append(idxs[i].topk(qs[i], 40, with_f64=True))

    _run_threads([lambda: worker(0), lambda: worker(1)])
    for i in range(2):
        for oi, _, cnt, o64 in outs[i]:
            np.testing.assert_array_equal(oi, expect[i][0])
            np.testing.assert_array_equal(o64, expect[i][3])
        idxs[i].close()
