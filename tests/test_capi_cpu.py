"""The C-ABI library loads and exports every function include/razorkv_b200.h declares (CPU;
no kernel is launched)."""

import os
import re

from razorkv_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _declared():
    with open(os.path.join(ROOT, "include", "razorkv_b200.h")) as f:
        src = f.read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rkv_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    assert "rkv_decode_attention" in names and "rkv_append_decode" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_binding_covers_every_declared_symbol():
    assert sorted(_lib.EXPORTED) == _declared()


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.rkv_abi_version() == 1
    assert lib.rkv_status_string(0) == b"ok"
    assert lib.rkv_status_string(4) == b"free page list exhausted"
    assert lib.rkv_workspace_error_flag_offset() == 0


def test_argument_errors_without_a_device():
    """Validation happens before any CUDA call, so bad arguments are reported on a CPU host."""
    lib = _lib.load()
    assert lib.rkv_select_pages(None, 1, 4, 2, None, None, None, 0, None) == 1
    assert lib.rkv_compact_pages(None, 0, 1, None, 1, 1, 1, None, 0, None) == 1
    assert lib.rkv_release_pages(None, 3, None, 0, None) == 1
    assert lib.rkv_page_salience_pool(None, 1, 8, 8, 4, 0, None, None) == 1


def test_zeroed_structures_are_rejected_not_crashed():
    """Every struct-taking entry point and size query survives zeroed or inconsistent
    structures (zero heads, zero page size, null pointers) and reports an error status or a
    zero size, without reaching CUDA."""
    lib = _lib.load()
    lay, q, o, s = _lib.KVLayout(), _lib.Query(), _lib.Output(), _lib.Salience()
    assert lib.rkv_decode_attention_workspace_size(q, lay) == 0
    assert lib.rkv_decode_fused_workspace_size(q, lay) == 0
    assert lib.rkv_decode_scored_workspace_size(q, lay) == 0
    assert lib.rkv_decode_attention(q, lay, 0.0, 0, o, None, 0, None) != 0
    assert lib.rkv_decode_attention_noalloc(q, lay, 0.0, 0, o, None) != 0
    assert lib.rkv_decode_fused(q, lay, s, 0.98, 0.02, 0.0, o, None, 0, None) != 0
    assert lib.rkv_decode_scored(q, q, lay, s, 0, 0.98, 0.02, 0.0, o, None, 0, None) != 0
    assert lib.rkv_append_decode(lay, s, None, None, 0, 0, None, None, 0, 0, q, 0.98, 0.02, 0.0,
                                 o, None, 0, None) != 0
    assert lib.rkv_score(q, lay, s, 0.98, 0.02, 1, None) != 0
    assert lib.rkv_gather_tokens(lay, 0, None, None, None, None) != 0
    assert lib.rkv_page_scores(lay, s, 0, 1, 16, None, None) != 0
    # a plausible layout whose page size is zero
    lay.k, lay.v, lay.dtype, lay.head_dim, lay.batch, lay.num_kv_heads = 16, 16, 2, 128, 1, 2
    assert lib.rkv_append(lay, s, 16, 16, 0, 0, 0, 1, 0, 16, 16, 4, 0, None) == 1
    q.q, q.dtype, q.num_heads, q.q_len = 16, 2, 3, 1   # 3 query heads over 2 kv heads
    assert lib.rkv_decode_attention_workspace_size(q, lay) > 0
    o.out, o.dtype = 16, 2
    assert lib.rkv_decode_attention(q, lay, 0.0, 0, o, None, 0, None) == 1


def test_integration_stub_matches_the_binding():
    """The ctypes stub printed in INTEGRATION.md declares the same structures as the
    package's binding (and include/razorkv_b200.h), so a maintainer who pastes it passes
    correctly laid-out arguments."""
    import ctypes
    with open(os.path.join(ROOT, "INTEGRATION.md")) as f:
        text = f.read()
    blocks = [b for b in re.findall(r"```python\n(.*?)```", text, flags=re.S)
              if "_paged_attention_cuda" in b]
    assert len(blocks) == 1
    src = blocks[0].replace('ctypes.CDLL("librazorkv_b200.so")', f'ctypes.CDLL({_lib.LIB_PATH!r})')
    ns = {}
    exec(compile(src, "INTEGRATION.md:stub", "exec"), ns)
    for stub, ours in ((ns["_KV"], _lib.KVLayout), (ns["_Q"], _lib.Query), (ns["_O"], _lib.Output)):
        assert [n for n, _ in stub._fields_] == [n for n, _ in ours._fields_]
        assert ctypes.sizeof(stub) == ctypes.sizeof(ours)
        for (n, _), (m, _) in zip(stub._fields_, ours._fields_):
            assert getattr(stub, n).offset == getattr(ours, m).offset
