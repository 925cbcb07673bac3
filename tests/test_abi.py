"""CPU: the C-ABI library loads, exports every symbol include/*.h declares,
and rejects bad arguments before touching the GPU."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT, package


def _declared():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names += re.findall(r"DSA_API\s+[\w\s\*]+?\b(dsa_\w+)\s*\(", open(h).read())
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    pkg = package()
    if not os.path.exists(pkg._lib.LIB_PATH):
        from importlib import import_module
        import_module(pkg.__name__ + ".build").build_cuda()
    return pkg._lib.load()


def test_header_declares_entry_points():
    names = _declared()
    for n in ("dsa_topk_indexer_launch", "dsa_topk_indexer_scores", "dsa_topk_indexer_partial",
              "dsa_topk_indexer_merge", "dsa_topk_indexer_status", "dsa_topk_indexer_error_string"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(package()._lib.LIB_PATH)
    for n in _declared():
        assert hasattr(raw, n), f"{n} declared in include/ but not exported"


def test_ctypes_signatures_cover_header(lib):
    assert {s[0] for s in package()._lib.SIGNATURES} == set(_declared())


def test_argument_errors_without_gpu(lib):
    P = ctypes.c_void_p
    ok = P(16)
    # null pointers / bad sizes are rejected before any CUDA call
    assert lib.dsa_topk_indexer_launch(None, ok, ok, ok, ok, ok, 4, 8, 16, None) == 1
    assert lib.dsa_topk_indexer_launch(ok, ok, ok, ok, ok, ok, -1, 8, 16, None) == 1
    assert lib.dsa_topk_indexer_launch(ok, ok, ok, ok, ok, ok, 4, 0, 16, None) == 1
    assert lib.dsa_topk_indexer_launch(P(17), ok, ok, ok, ok, ok, 4, 8, 16, None) == 2
    assert lib.dsa_topk_indexer_scores(ok, ok, ok, ok, ok, ok, 10, 4, 8, 16, None) == 1  # stride < 8*64
    assert lib.dsa_topk_indexer_partial(ok, ok, ok, ok, ok, 10, 5, ok, ok, 4, 8, 16, None) == 1
    assert lib.dsa_topk_indexer_merge(ok, ok, 0, ok, ok, ok, 4, 8, None) == 1
    # empty batch is a no-op
    assert lib.dsa_topk_indexer_launch(None, None, None, None, None, None, 0, 8, 16, None) == 0
    assert b"aligned" in lib.dsa_topk_indexer_error_string(2)


def test_torch_wrapper_validates_before_launch(pkg):
    import torch
    q = torch.zeros((2, 64, 128), dtype=torch.uint8)
    kc = torch.zeros((4, 64, 1, 132), dtype=torch.uint8)
    w = torch.zeros((2, 64))
    sl = torch.zeros(2, dtype=torch.int32)
    bt = torch.zeros((2, 2), dtype=torch.int32)
    out = torch.zeros((2, 2048), dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        pkg.launch_topk_c(q, kc, w, sl, bt, out)


def test_missing_library_fails_loudly(monkeypatch):
    """No CPU fallback: without the built CUDA library every entry point
    raises instead of computing something else."""
    import torch
    pkg = package()
    monkeypatch.setattr(pkg._lib, "LIB_PATH", os.path.join(ROOT, "no-such-dir", "libdsa_topk_indexer.so"))
    monkeypatch.setattr(pkg._lib, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        pkg._lib.load()
    with pytest.raises(RuntimeError):
        pkg.last_launch_count()


def test_queue_constants_match_header():
    """The decode-queue record constants of the Python binding equal the
    header's #defines (the record is built on the host, read on the GPU)."""
    text = open(os.path.join(ROOT, "include", "dsa_topk_indexer.h")).read()
    defs = dict(re.findall(r"#define\s+(DSA_(?:QUEUE|STATUS)_\w+)\s+(0x[0-9a-f]+|\d+)u?", text))
    lib = package()._lib
    for name, val in defs.items():
        assert getattr(lib, name) == int(val, 0), name


def test_queue_apply_argument_errors(lib):
    P = ctypes.c_void_p
    ok = P(16)
    assert lib.dsa_decode_queue_apply(None, 64, ok, ok, 4, 8, ok, ok, 4, None) == 1
    assert lib.dsa_decode_queue_apply(ok, 4, ok, ok, 4, 8, ok, ok, 4, None) == 1   # record below the header
    assert lib.dsa_decode_queue_apply(ok, 64, ok, ok, 0, 8, ok, ok, 4, None) == 1  # no slots
    assert lib.dsa_decode_queue_apply(ok, 64, ok, ok, 4, 8, ok, ok, 0, None) == 1  # no batch rows


def test_peer_merge_argument_errors(lib):
    """The peer-exchange entry points reject bad arguments before any CUDA
    call (no GPU needed)."""
    P = ctypes.c_void_p
    ok = P(16)
    n = ctypes.c_int64(0)
    assert lib.dsa_peer_region_bytes(0, ctypes.byref(n)) == 1
    assert lib.dsa_peer_region_bytes(4, ctypes.byref(n)) == 0 and n.value == 3 * 4 * 2048 * 4 + 512
    assert lib.dsa_peer_merge(None, 2, 0, 1, 4, ok, 8, 15, 0, None) == 1   # no bases
    assert lib.dsa_peer_merge(ok, 0, 0, 1, 4, ok, 8, 15, 0, None) == 1     # no ranks
    assert lib.dsa_peer_merge(ok, 2, 2, 1, 4, ok, 8, 15, 0, None) == 1     # rank >= nranks
    assert lib.dsa_peer_merge(ok, 65, 0, 1, 4, ok, 8, 15, 0, None) == 1    # more than 64 ranks
    assert lib.dsa_peer_merge(ok, 2, 0, 1, 4, ok, 8, 16, 0, None) == 1     # unknown phase bit
    assert lib.dsa_peer_alloc(0, ctypes.byref(P()), ctypes.create_string_buffer(64)) == 1
    assert lib.dsa_peer_open(None, ctypes.byref(P())) == 1
