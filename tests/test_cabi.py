"""The C-ABI library loads and exports every symbol include/imi_b200.h declares
(no compute calls: runs without a GPU)."""
import ctypes
import re
from pathlib import Path

from adaptiveimi_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "imi_b200.h").read_text()
    return sorted(set(re.findall(r"^IMI_API\s+[\w\s\*]+?\b(imi_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 9
    for s in syms:
        assert hasattr(L, s), s
    assert set(syms) == set(_lib.EXPORTS)
    assert L.imi_abi_version() == 2


def test_descriptor_sizes_match_header():
    # field counts of the ctypes mirrors against the C struct bodies
    text = (ROOT / "include" / "imi_b200.h").read_text()
    for cname, py in (("imi_build_desc", _lib.BuildDesc), ("imi_select_desc", _lib.SelectDesc),
                      ("imi_attn_desc", _lib.AttnDesc), ("imi_append_desc", _lib.AppendDesc),
                      ("imi_async_desc", _lib.AsyncDesc), ("imi_apply_desc", _lib.ApplyDesc),
                      ("imi_merge_desc", _lib.MergeDesc), ("imi_combine_desc", _lib.CombineDesc),
                      ("imi_peer_gather_desc", _lib.PeerGatherDesc)):
        body = re.search(r"typedef struct " + cname + r" \{(.*?)\} " + cname, text, re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        names = re.findall(r"\*?\s*(\w+)(?:\[\d+\])?\s*[,;]", body)
        assert [f[0] for f in py._fields_] == names, cname


def test_workspace_query_and_invalid_args_without_gpu():
    L = _lib.load()
    ks = (ctypes.c_int32 * 4)(90, 90, 1, 1)
    ws = L.imi_build_workspace_size(8, 130976, 128, 2, ctypes.cast(ks, ctypes.c_void_p))
    assert ws > 8 * 130976 * 4
    # a null descriptor is rejected with a message, before touching CUDA
    assert L.imi_select_cells(None, None) != 0
    assert b"null descriptor" in L.imi_last_error()


def test_sequence_sharding_entries_reject_bad_descriptors_without_gpu():
    L = _lib.load()
    # peer exchange: every check happens before any launch
    d = _lib.PeerGatherDesc()
    assert L.imi_peer_allgather(ctypes.byref(d), None) != 0
    assert b"null pointer" in L.imi_last_error()
    buf = (ctypes.c_uint64 * 8)()
    addr = ctypes.addressof(buf)
    d.src_peers = d.flag_peers = d.epoch = d.ticket = d.dst = addr
    d.world, d.rank, d.bytes = 2, 2, 64  # rank out of range
    assert L.imi_peer_allgather(ctypes.byref(d), None) != 0
    assert b"rank < world" in L.imi_last_error()
    d.rank, d.bytes = 1, 24  # not a multiple of 16
    assert L.imi_peer_allgather(ctypes.byref(d), None) != 0
    # merge and combine
    m = _lib.MergeDesc()
    assert L.imi_merge_candidates(ctypes.byref(m), None) != 0
    assert b"null pointer" in L.imi_last_error()
    c = _lib.CombineDesc()
    assert L.imi_combine_partials(ctypes.byref(c), None) != 0
    assert b"null pointer" in L.imi_last_error()
