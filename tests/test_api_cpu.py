"""Host-side checks without a GPU: the C ABI library loads and exports everything
include/tiso.h declares; its size queries and argument checks; the public API's validation
(the reference's error types and messages, tests/test_isotonic.py:143-165) and its refusal of
CPU tensors (no CPU fallback)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import torchisotonic_b200
from torchisotonic_b200 import _ext

HEADER = Path(__file__).resolve().parent.parent / "include" / "tiso.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(tiso_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol() -> None:
    names = declared()
    assert {"tiso_fit", "tiso_grad", "tiso_fit_workspace_size", "tiso_grad_workspace_size",
            "tiso_last_error", "tiso_abi_version"} <= set(names)
    so = _ext.lib()
    for name in names:
        assert hasattr(so, name), name
    assert so.tiso_abi_version() == _ext.ABI_VERSION


def test_workspace_queries() -> None:
    so = _ext.lib()
    size = ctypes.c_size_t()
    assert so.tiso_fit_workspace_size(_ext.F32, 0, 1_000_000, 16, _ext.EXACT, ctypes.byref(size)) == 0
    assert size.value == 0  # short rows: one launch, no scratch
    assert so.tiso_fit_workspace_size(_ext.F32, 1, 1, 100_000_000, _ext.EXACT,
                                      ctypes.byref(size)) == 0
    assert size.value >= 100_000_000 * 20  # a block slot per element, worst case
    assert so.tiso_grad_workspace_size(_ext.F64, 1, 4096, 65536, 0, ctypes.byref(size)) == 0
    assert size.value > 0


def test_argument_errors() -> None:
    so = _ext.lib()
    size = ctypes.c_size_t()
    assert so.tiso_fit_workspace_size(7, 0, 1, 16, 0, ctypes.byref(size)) == 1
    assert b"dtype" in so.tiso_last_error()
    assert so.tiso_fit_workspace_size(_ext.F32, 0, 1, 0, 0, ctypes.byref(size)) == 1
    assert so.tiso_fit_workspace_size(_ext.F32, 0, 1, 2**31, 0, ctypes.byref(size)) == 1
    assert b"2^31" in so.tiso_last_error()
    # a long row without its workspace is refused before any launch
    rc = so.tiso_fit(_ext.F32, ctypes.c_void_p(16), None, ctypes.c_void_p(16), None, 1, 10_000,
                     _ext.EXACT, 0.0, 0.0, None, None, 0, None)
    assert rc == 2 and b"workspace" in so.tiso_last_error()
    # the weights' gradient needs w, y and grad_w
    rc = so.tiso_grad(_ext.F32, None, None, ctypes.c_void_p(16), ctypes.c_void_p(16), None, None,
                      1, 16, _ext.WANT_GRAD_W, 0.0, 0.0, None, 0, None)
    assert rc == 1


def test_bad_inputs() -> None:
    iso = torchisotonic_b200.isotonic
    with pytest.raises(TypeError, match=r"y must be a torch\.Tensor, got list"):
        iso([1.0, 2.0])  # type: ignore[arg-type]
    with pytest.raises(TypeError, match="complex"):
        iso(torch.zeros(3, dtype=torch.complex64))
    with pytest.raises(ValueError, match="at least one dimension"):
        iso(torch.tensor(1.0))
    with pytest.raises(TypeError, match=r"weight must be a torch\.Tensor"):
        iso(torch.zeros(3), [1.0, 1.0, 1.0])  # type: ignore[arg-type]
    with pytest.raises(ValueError, match="does not fit y"):
        iso(torch.zeros(3), torch.ones(4))


@pytest.mark.parametrize("shape", [(0,), (3, 0), (0, 5)])
def test_empty(shape: tuple[int, ...]) -> None:
    got = torchisotonic_b200.isotonic(torch.empty(shape))
    assert got.shape == shape
    assert torchisotonic_b200.isotonic(torch.empty(shape, dtype=torch.int64)).dtype == \
        torch.get_default_dtype()


def test_cpu_tensors_are_refused() -> None:
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        torchisotonic_b200.isotonic(torch.tensor([3.0, 1.0, 2.0]))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        _ext.isotonic_tiles(torch.zeros(2, 3), None, True)


def test_no_oracle_in_the_product_path() -> None:
    # The package imports nothing from the oracle (test infrastructure only).
    pkg = Path(torchisotonic_b200.__file__).resolve().parent
    for f in list(pkg.glob("*.py")) + list((pkg / "csrc").glob("*")):
        if f.suffix == ".so":
            continue
        text = f.read_text()
        assert "import oracle" not in text and "from oracle" not in text, f
        assert "oracle/" not in text and "liboracle" not in text, f


def test_varlen_refusals() -> None:
    so = _ext.lib()
    # max_len over the limit, and a missing offsets array, are refused before any launch
    rc = so.tiso_fit_varlen(_ext.F32, ctypes.c_void_p(16), None, ctypes.c_void_p(16), None,
                            ctypes.c_void_p(16), 3, 513, _ext.EXACT, 0.0, 0.0, None, None)
    assert rc == 1 and b"512" in so.tiso_last_error()
    rc = so.tiso_fit_varlen(_ext.F32, ctypes.c_void_p(16), None, ctypes.c_void_p(16), None, None,
                            3, 16, _ext.EXACT, 0.0, 0.0, None, None)
    assert rc == 1 and b"offsets" in so.tiso_last_error()
    rc = so.tiso_grad_varlen(_ext.F32, None, None, ctypes.c_void_p(16), ctypes.c_void_p(16), None,
                             None, ctypes.c_void_p(16), 3, 16, _ext.WANT_GRAD_W, 0.0, 0.0, None)
    assert rc == 1
    # nothing to do: no rows, or only empty ones
    assert so.tiso_fit_varlen(_ext.F32, None, None, None, None, None, 0, 0, 0, 0.0, 0.0, None,
                              None) == 0
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        torchisotonic_b200.isotonic_varlen(torch.zeros(4), torch.tensor([0, 2, 4]))
    with pytest.raises(TypeError, match="integer"):
        torchisotonic_b200.isotonic_varlen(torch.zeros(4), torch.tensor([0.0, 4.0]))
    with pytest.raises(ValueError, match="1-D"):
        torchisotonic_b200.isotonic_varlen(torch.zeros(2, 2), torch.tensor([0, 4]))


def test_operator_schemas_follow_the_reference() -> None:
    # the reference's schemas (src/torchisotonic/csrc/ops.cpp:47-50), under this library's
    # namespace; fake kernels propagate shapes without a GPU (meta tensors)
    from torchisotonic_b200 import ops  # noqa: F401 - registers the operators

    schemas = {
        "isotonic_tiles": "(Tensor y, Tensor? w, bool increasing, bool exact=True, "
                          "bool with_starts=False) -> Tensor[]",
        "isotonic_grad": "(Tensor out, Tensor starts, Tensor g, Tensor? w, Tensor? y) -> Tensor[]",
    }
    for name, sig in schemas.items():
        op = getattr(torch.ops.torchisotonic_b200, name).default
        assert str(op._schema) == f"torchisotonic_b200::{name}{sig}"
    y = torch.empty(3, 5, device="meta")
    out, st = torch.ops.torchisotonic_b200.fit(y, None, True, True, True, None, 1.0)
    assert out.shape == (3, 5) and st.shape == (3, 5) and st.dtype == torch.bool
    out, st = torch.ops.torchisotonic_b200.isotonic_tiles(y, None, True)
    assert out.shape == (3, 5) and st.numel() == 0
    gy, gw = torch.ops.torchisotonic_b200.isotonic_grad(y, y.bool(), y, y, y)
    assert gy.shape == (3, 5) and gw.shape == (3, 5)
    gy, gw = torch.ops.torchisotonic_b200.fit_grad(y.bool(), y, None, None, True, False, None, None)
    assert gy.shape == (3, 5) and gw.numel() == 0
