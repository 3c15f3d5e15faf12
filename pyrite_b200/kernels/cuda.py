"""Device-resident fused dequantize x matvec (weights in HBM, fp32 activations).

The B200 counterpart of the executor's row-range call
``_matrix_matvec(name, first_row, row_count, vector)`` (reference
``pyrite/executor.py:481-509``): a :class:`QuantMatrix` holds one GGML matrix in
device memory and multiplies any block-aligned row range of it by one or more
fp32 columns, on the caller's current stream.  PyTorch supplies only device
memory and streams; the arithmetic is in libpyrite_b200.so.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib
from ..ggml_types import spec


def _stream_handle(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _check(code: int, what: str) -> None:
    if code == -4:
        raise RuntimeError(f"{what}: CUDA error ({_lib.error_string(code)})")
    if code != 0:
        raise ValueError(f"{what} rejected the matrix buffer/shape (error {code}: {_lib.error_string(code)})")


STATIC_WEIGHTS = 1  # PYRITE_F_STATIC_WEIGHTS


def matvec(ggml_type: int, weights: torch.Tensor, x: torch.Tensor, rows: int, cols: int,
           out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
           static_weights: bool = False, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``out[c, r] = sum_k W[r, k] x[c, k]`` for a device payload of ``rows`` rows.

    ``weights``: contiguous uint8 CUDA tensor of exactly ``rows * row_bytes``
    bytes.  ``x``: float32 CUDA tensor ``(cols,)`` or ``(ncols, cols)`` with unit
    stride along ``cols``.  Returns ``(rows,)`` or ``(ncols, rows)`` float32.
    ``static_weights``: the payload is not written by the kernel just before
    this call on the stream, so its weight stream may overlap that kernel.
    ``workspace``: uint8 CUDA tensor of at least ``workspace_size(...) + 256``
    bytes for the re-encoded activation (allocated per call when omitted).
    """
    lib = _lib.require()
    if weights.dtype != torch.uint8 or not weights.is_cuda or not weights.is_contiguous():
        raise ValueError("weights must be a contiguous uint8 CUDA tensor")
    if x.dtype != torch.float32 or not x.is_cuda or x.device != weights.device:
        raise ValueError("x must be a float32 tensor on the weights' device")
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if x2.dim() != 2 or x2.shape[1] != cols or x2.stride(1) != 1:
        raise ValueError("matrix/vector shape mismatch")
    ncols = x2.shape[0]
    if out is None:
        out2 = torch.empty((ncols, rows), dtype=torch.float32, device=x.device)
    else:
        out2 = out.unsqueeze(0) if out.dim() == 1 else out
        if out2.shape != (ncols, rows) or out2.stride(1) != 1 or out2.dtype != torch.float32:
            raise ValueError("out has the wrong shape, dtype or layout")
    if workspace is None:
        workspace = torch.empty(int(lib.pyrite_cuda_workspace_size(ggml_type, cols, ncols)) + 256,
                                dtype=torch.uint8, device=x.device)
    ws_ptr = workspace.data_ptr()
    ws_off = (-ws_ptr) % 256
    code = lib.pyrite_cuda_matvec(ggml_type, weights.data_ptr(), weights.numel(), x2.data_ptr(),
                                  x2.stride(0) if ncols > 1 else cols, out2.data_ptr(),
                                  out2.stride(0) if ncols > 1 else rows, rows, cols, ncols,
                                  STATIC_WEIGHTS if static_weights else 0, ws_ptr + ws_off,
                                  workspace.numel() - ws_off, _stream_handle(stream))
    _check(code, "cuda matvec")
    return out2[0] if squeeze else out2


@dataclass
class PreparedX:
    """An activation re-encoded once for several matvecs (see prepare_x)."""

    x: torch.Tensor          # (cols,) float32
    workspace: torch.Tensor  # uint8, the encoding
    offset: int              # 256-byte alignment offset inside workspace

    @property
    def ptr(self) -> int:
        return self.workspace.data_ptr() + self.offset

    @property
    def nbytes(self) -> int:
        return self.workspace.numel() - self.offset


def prepare_x(x: torch.Tensor, workspace: torch.Tensor | None = None,
              stream: torch.cuda.Stream | None = None) -> PreparedX:
    """Encode one fp32 activation for :func:`matvec_prepared` (enqueued on the stream)."""
    lib = _lib.require()
    if x.dtype != torch.float32 or not x.is_cuda or x.dim() != 1 or x.stride(0) != 1:
        raise ValueError("x must be a contiguous 1-D float32 CUDA tensor")
    cols = x.shape[0]
    need = int(lib.pyrite_cuda_workspace_size(0, cols, 1)) + 256
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    off = (-workspace.data_ptr()) % 256
    code = lib.pyrite_cuda_prepare_x(x.data_ptr(), cols, cols, 1, workspace.data_ptr() + off,
                                     workspace.numel() - off, _stream_handle(stream))
    _check(code, "prepare_x")
    return PreparedX(x, workspace, off)


def matvec_prepared(ggml_type: int, weights: torch.Tensor, px: PreparedX, rows: int, cols: int,
                    out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
                    static_weights: bool = False) -> torch.Tensor:
    """``out[r] = sum_k W[r, k] x[k]`` with x encoded earlier by :func:`prepare_x`."""
    lib = _lib.require()
    if weights.dtype != torch.uint8 or not weights.is_cuda or not weights.is_contiguous():
        raise ValueError("weights must be a contiguous uint8 CUDA tensor")
    if px.x.shape[0] != cols:
        raise ValueError("matrix/vector shape mismatch")
    if out is None:
        out = torch.empty(rows, dtype=torch.float32, device=weights.device)
    elif out.shape != (rows,) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out has the wrong shape, dtype or layout")
    code = lib.pyrite_cuda_matvec_prepared(ggml_type, weights.data_ptr(), weights.numel(), px.x.data_ptr(),
                                           px.ptr, px.nbytes, out.data_ptr(), rows, cols,
                                           STATIC_WEIGHTS if static_weights else 0, _stream_handle(stream))
    _check(code, "cuda matvec")
    return out


def workspace_size(ggml_type: int, cols: int, ncols: int = 1) -> int:
    """Bytes of device workspace a matvec needs (pass 256 more for alignment)."""
    return int(_lib.require().pyrite_cuda_workspace_size(ggml_type, cols, ncols))


def dequantize_rows(ggml_type: int, weights: torch.Tensor, rows: int, cols: int,
                    out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Decode ``rows x cols`` values to fp32 (each the rounded reference fp64 value)."""
    lib = _lib.require()
    if weights.dtype != torch.uint8 or not weights.is_cuda or not weights.is_contiguous():
        raise ValueError("weights must be a contiguous uint8 CUDA tensor")
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.float32, device=weights.device)
    elif out.shape != (rows, cols) or not out.is_contiguous() or out.dtype != torch.float32:
        raise ValueError("out has the wrong shape, dtype or layout")
    code = lib.pyrite_cuda_dequantize_rows(ggml_type, weights.data_ptr(), weights.numel(), out.data_ptr(),
                                           rows, cols, _stream_handle(stream))
    _check(code, "cuda dequantize")
    return out


def status(clear: bool = True) -> int:
    """Device status word (bit 0: a kernel timed out waiting for a copy)."""
    return int(_lib.require().pyrite_cuda_status(1 if clear else 0))


@dataclass
class QuantMatrix:
    """One GGML matrix resident in HBM: ``rows`` rows of ``cols`` values."""

    ggml_type: int
    rows: int
    cols: int
    data: torch.Tensor  # uint8, rows * row_bytes
    static: bool = True  # resident weights are never rewritten by the kernels that precede a matvec

    @property
    def row_bytes(self) -> int:
        s = spec(self.ggml_type)
        return self.cols // s.block_size * s.bytes_per_block

    @classmethod
    def from_bytes(cls, ggml_type: int, payload, rows: int, cols: int, device="cuda") -> "QuantMatrix":
        t = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
        return cls(ggml_type, rows, cols, t.to(device))

    def row_range(self, first_row: int, row_count: int) -> torch.Tensor:
        """Byte view of rows [first_row, first_row + row_count)."""
        if first_row < 0 or row_count < 0 or first_row + row_count > self.rows:
            raise ValueError(f"row range [{first_row}, {first_row + row_count}) outside the matrix")
        rb = self.row_bytes
        return self.data[first_row * rb:(first_row + row_count) * rb]

    def matvec(self, x: torch.Tensor, first_row: int = 0, row_count: int | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
        n = self.rows - first_row if row_count is None else row_count
        return matvec(self.ggml_type, self.row_range(first_row, n), x, n, self.cols, out=out,
                      static_weights=self.static)

    def dequantize(self, first_row: int = 0, row_count: int = 1) -> torch.Tensor:
        return dequantize_rows(self.ggml_type, self.row_range(first_row, row_count), row_count, self.cols)
