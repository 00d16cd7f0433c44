"""CPU-only checks of the C ABI library: it loads, exports every declared
symbol, validates arguments before touching the GPU, and maps errors to the
reference's Python exception types."""

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "maxsim_b200.h"


def _declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(msb_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_loads():
    from maxsim_b200 import _lib

    assert _lib.LIB_PATH.exists()
    assert _lib.lib.msb_version() == 1


def test_every_declared_symbol_is_exported_and_bound():
    from maxsim_b200 import _lib

    declared = _declared_symbols()
    assert declared, "no msb_ symbols found in the header"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\b(msb_[a-z0-9_]+)\b", out))
    missing = [s for s in declared if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    unbound = [s for s in declared if s not in _lib.SIGNATURES]
    assert not unbound, f"declared but not bound in _lib.SIGNATURES: {unbound}"


def test_option_errors_map_to_value_error():
    from maxsim_b200 import _lib

    with pytest.raises(ValueError, match="unknown option"):
        _lib.check(_lib.lib.msb_set_option(b"no_such_option", 1))
    with pytest.raises(ValueError, match="engine must be"):
        _lib.set_engine(7)
    assert _lib.get_engine() in (0, 1, 2)


@pytest.mark.parametrize("name,default", [("tc_int8_cache", 1), ("tc_f16_cache", 0), ("tc_row_replicas", 1),
                                          ("tc_fused_topk", 0)])
def test_boolean_options_round_trip(name, default):
    """Every tensor-core routing option reads back what was set, defaults as documented, and refuses values
    other than 0 and 1."""
    from maxsim_b200 import _lib

    assert _lib.get_option(name) == default
    try:
        for v in (1 - default, default):
            _lib.set_option(name, v)
            assert _lib.get_option(name) == v
        with pytest.raises(ValueError, match=f"{name} must be 0 or 1"):
            _lib.set_option(name, 2)
    finally:
        _lib.set_option(name, default)


def test_handle_validation_happens_before_device_work():
    """Offsets / scale errors are ValueError (reference std::invalid_argument)."""
    from maxsim_b200 import _maxsim_cuda as mc

    packed = np.zeros((3, 64), np.uint8)
    with pytest.raises(ValueError, match="offsets must start at 0"):
        mc.CudaInt4PackedDocs(packed, np.array([1, 3], np.int64), 128, 1.0)
    with pytest.raises(ValueError, match="offsets must end at num_doc_tokens"):
        mc.CudaInt4PackedDocs(packed, np.array([0, 2], np.int64), 128, 1.0)
    with pytest.raises(ValueError, match="nondecreasing"):
        mc.CudaInt4PackedDocs(packed, np.array([0, 2, 1, 3], np.int64), 128, 1.0)
    with pytest.raises(ValueError, match="scale must be finite"):
        mc.CudaInt4PackedDocs(packed, np.array([0, 3], np.int64), 128, 0.0)
    with pytest.raises(ValueError, match="packed shape does not match dim"):
        mc.CudaInt4PackedDocs(packed, np.array([0, 3], np.int64), 64, 1.0)
    with pytest.raises(ValueError, match="divisible by 8"):
        mc.CudaPackedDocs(np.zeros((3, 1), np.uint8), np.array([0, 3], np.int64), 12)


def test_ctypes_structs_match_header_layout(tmp_path):
    """Compile the header with gcc and compare struct sizes / offsets with the ctypes mirror."""
    from maxsim_b200 import _lib

    src = tmp_path / "layout.c"
    fields_o = [name for name, _ in _lib.ScoreOpts._fields_]
    fields_i = [name for name, _ in _lib.DocsInfo._fields_]
    body = ['#include <stdio.h>', '#include <stddef.h>', '#include "maxsim_b200.h"', "int main(void){",
            'printf("%zu %zu\\n", sizeof(msb_score_opts), sizeof(msb_docs_info));']
    body += [f'printf("%zu\\n", offsetof(msb_score_opts, {f}));' for f in fields_o]
    body += [f'printf("%zu\\n", offsetof(msb_docs_info, {f}));' for f in fields_i]
    body += ["return 0;}"]
    src.write_text("\n".join(body))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", f"-I{REPO / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert int(lines[0]) == ctypes.sizeof(_lib.ScoreOpts)
    assert int(lines[1]) == ctypes.sizeof(_lib.DocsInfo)
    offs = [int(x) for x in lines[2:]]
    assert offs[: len(fields_o)] == [getattr(_lib.ScoreOpts, f).offset for f in fields_o]
    assert offs[len(fields_o):] == [getattr(_lib.DocsInfo, f).offset for f in fields_i]


def test_cpu_device_requests_fail_loudly():
    import maxsim_b200 as m

    docs = np.ones((2, 8), np.float32)
    packed = m.pack_signs(docs)
    with pytest.raises(NotImplementedError, match="GPU only"):
        m.maxsim(np.ones((1, 8), np.float32), packed, device="cpu")
    idx = m.Index.from_embeddings(["a", "b"], np.ones((2, 128), np.float32), np.array([0, 1, 2]), mode="int4")
    with pytest.raises(NotImplementedError, match="GPU only"):
        m.Reranker(idx, device="cpu")


def test_score_options_take_host_arrays_or_tensor_pointers():
    """The option struct carries a numpy array's address for the synchronous calls and a tensor's
    data_ptr for the *_device calls (which need device memory there)."""
    import numpy as np
    import torch

    from maxsim_b200._maxsim_cuda import _opts

    w = np.arange(4, dtype=np.float32)
    t = torch.arange(4, dtype=torch.float32)
    assert _opts(reducer=1, weights=w).weights == w.ctypes.data
    assert _opts(reducer=1, weights=t).weights == t.data_ptr()
    assert _opts(override=t).doc_scale_override == t.data_ptr()
    o = _opts()
    assert not o.weights and not o.doc_scale_override
