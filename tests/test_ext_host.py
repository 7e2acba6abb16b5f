"""Host-side behaviour of tilec_b200.ext.matrix_mul that needs no GPU.

Mirrors the reference's error behaviour (tilec/ext.py:55-58, tilec/jit.py:34-39) and
checks that there is no CPU fallback.
"""
import pytest
import torch

from tilec_b200 import ext
from tilec_b200.language import cdiv


def test_shape_mismatch_message_matches_reference():
    x1, x2 = torch.zeros(3, 4), torch.zeros(5, 2)
    with pytest.raises(ValueError, match=r"^matrix_mul: shapes \(3, 4\) and \(5, 2\) don't match$"):
        ext.matrix_mul(x1, x2)


def test_shape_error_comes_before_dtype_error():
    # The reference checks shapes (ext.py:57) before it type-checks kernel arguments (jit.py:34).
    with pytest.raises(ValueError):
        ext.matrix_mul(torch.zeros(3, 4, dtype=torch.float64), torch.zeros(5, 2, dtype=torch.float64))


@pytest.mark.parametrize("bad", [torch.zeros(2, 3, 4), torch.zeros(3)])
def test_non_2d_inputs_raise_value_error(bad):
    with pytest.raises(ValueError):
        ext.matrix_mul(bad, torch.zeros(3, 3))
    with pytest.raises(ValueError):
        ext.matrix_mul(torch.zeros(3, 3), bad)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float16, torch.bfloat16, torch.int32])
def test_non_fp32_raises_type_error(dtype):
    with pytest.raises(TypeError, match="float32"):
        ext.matrix_mul(torch.zeros(2, 3, dtype=dtype), torch.zeros(3, 2, dtype=dtype))


def test_cpu_tensors_raise_no_fallback():
    with pytest.raises(ValueError, match="CUDA"):
        ext.matrix_mul(torch.zeros(2, 3), torch.zeros(3, 2))


def test_bad_variant_name():
    from tilec_b200 import _native
    with pytest.raises(ValueError, match="unknown matrix_mul variant"):
        _native.make_cfg("fastest")


def test_operand_views_pass_through():
    x = torch.zeros(8, 10)
    v = x[:, 2:7]  # unit column stride, row stride 10: passed through, ld = 10
    t, ld, trans = ext._operand(v)
    assert t.data_ptr() == v.data_ptr() and ld == 10 and not trans
    # transposed view: passed as transposed storage (the reference copies, ext.py:59-60)
    t, ld, trans = ext._operand(x.t())
    assert t.data_ptr() == x.data_ptr() and ld == 10 and trans
    t, ld, trans = ext._operand(x[1:7, 2:9].t())  # transposed sub-view: ld = row stride of x
    assert t.data_ptr() == x[1:7, 2:9].data_ptr() and ld == 10 and trans
    t, ld, trans = ext._operand(torch.zeros(1, 5).expand(4, 5))  # overlapping rows: copied
    assert t.is_contiguous() and ld == 5 and not trans
    t, ld, trans = ext._operand(x[::2, ::3])  # no unit stride: copied
    assert t.is_contiguous() and ld == 4 and not trans


def test_cdiv_and_configs():
    assert cdiv(5000, 4096) == 2 and cdiv(0, 64) == 0
    cfgs = ext.kernel_configs(512, 4096, 64)
    assert ("simt", 1) in cfgs and ("3xtf32", 1) in cfgs
    assert all(v in ("simt", "splitk", "tf32", "3xtf32") for v, _ in cfgs)
    # misaligned shapes still get tensor-core candidates (their operands are packed first)
    assert ("3xtf32", 1) in ext.kernel_configs(1000, 3001, 777)


@pytest.mark.parametrize("M,chunks", [(65536, 8), (65536, 16), (8192, 3), (4096, 4), (1000, 8), (300, 2), (1, 8),
                                      (100000, 7)])
def test_row_chunks_cover_rows_in_order(M, chunks):
    spans = ext._row_chunks(M, chunks)
    assert spans[0][0] == 0 and spans[-1][1] == M
    assert all(a < b for a, b in spans)
    assert all(spans[i][1] == spans[i + 1][0] for i in range(len(spans) - 1))
    # every span but the last starts on a 256-row (CTA-pair tile) boundary
    assert all(a % 256 == 0 for a, _ in spans)


def test_row_chunks_taper_both_ends():
    sizes = [b - a for a, b in ext._row_chunks(65536, 8)]
    assert sizes[:3] == [2048, 2048, 4096] and sizes[-3:] == [4096, 2048, 2048]
    assert set(sizes[3:-3]) == {8192}
    assert [b - a for a, b in ext._row_chunks(65536, 8, taper=False)] == [8192] * 8


def test_row_chunks_explicit_sizes():
    assert ext._row_chunks(10, [3, 7]) == [(0, 3), (3, 10)]
    with pytest.raises(ValueError):
        ext._row_chunks(10, [3, 6])
    with pytest.raises(ValueError):
        ext._row_chunks(10, [0, 10])
