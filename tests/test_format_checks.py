"""The Python wrappers refuse weights whose layout does not match K before any launch: the kernels read whole rows of
K through raw pointers (as the C ABI's callers must guarantee), so a mismatch would read past the tensors. CPU only."""

import pytest
import torch

from locals_b200.kernels import _check_format


def _w(rows, K, bits, lead=()):
    return (torch.zeros((*lead, rows, K * bits // 32), dtype=torch.int32),
            torch.zeros((*lead, rows, K // 64), dtype=torch.bfloat16),
            torch.zeros((*lead, rows, K // 64), dtype=torch.bfloat16))


@pytest.mark.parametrize("bits", [4, 8])
def test_matching_layouts_pass(bits):
    _check_format(*_w(96, 2048, bits), 2048, bits, 64)
    _check_format(*_w(2048, 768, bits, lead=(64,)), 768, bits, 64)  # a stacked (E, N, ...) expert matrix


def test_wrong_k_is_refused():
    with pytest.raises(ValueError):
        _check_format(*_w(2048, 768, 4, lead=(64,)), 2048, 4, 64)  # an (E, D, I/8) down stack fed D-wide rows
    with pytest.raises(ValueError):
        _check_format(*_w(96, 2048, 4), 2048, 8, 64)  # 4-bit words read as 8-bit
    with pytest.raises(ValueError):
        _check_format(*_w(96, 2048, 4), 2000, 4, 64)  # K not a multiple of the group


def test_rows_must_agree():
    w, s, b = _w(96, 2048, 4)
    with pytest.raises(ValueError):
        _check_format(w, s[:48], b[:48], 2048, 4, 64)
    with pytest.raises(ValueError):
        _check_format(w, s, b[:, :16], 2048, 4, 64)
