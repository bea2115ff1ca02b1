"""The drop-in boundary without a GPU: the C-ABI library builds, loads and
exports every function include/wpt_attn.h declares, the ctypes table
declares the same set, and the host-side logic of the kernel-form module
(column counts, tree masks, kernel choice, refusal of CPU tensors) follows
the reference's contract (pytorch_kernels.py:18-26,73-77)."""

import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "wpt_attn.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wpt_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def library():
    from wpt_b200 import build
    build.build()
    return ctypes.CDLL(build.TARGET)


def test_library_exports_every_declared_symbol(library):
    names = _declared()
    assert "wpt_attn_prefill" in names and "wpt_accept" in names
    for name in names:
        assert hasattr(library, name), name


def test_ctypes_table_matches_the_header():
    from wpt_b200 import _lib
    assert sorted(_lib.SIGNATURES) == _declared()


def test_last_error_is_callable_without_a_gpu(library):
    library.wpt_last_error.restype = ctypes.c_char_p
    assert isinstance(library.wpt_last_error(), bytes)


def test_invalid_shapes_are_refused_before_any_launch(library):
    # argument checks run on the host: an unsupported head width is WPT_ERR_UNSUPPORTED (2)
    from wpt_b200 import _lib
    lib = _lib.lib()
    rc = lib.wpt_attn_prefill(None, None, None, 0, 0, 0, 0, None, None, None, None, None, None, None, None, None, 1,
                              1, 1, 1, 96, 1, 0, 1.0, None)
    assert rc == _lib.ERR_UNSUPPORTED
    with pytest.raises(NotImplementedError, match="head width 96"):
        _lib.check(rc)


def test_chosen_columns_follows_the_reference():
    import wpt_b200
    assert wpt_b200.chosen_columns(1024, 128, 100) == 0
    assert wpt_b200.chosen_columns(1024, 128, 500) == 372
    assert wpt_b200.chosen_columns(1024, 128, 5000) == 1024


def test_tree_of_more_than_64_nodes_is_refused_before_any_launch():
    from wpt_b200 import ops
    with pytest.raises(NotImplementedError):
        ops.tree_bits(torch.arange(65) - 1, 1)  # refused on the host, before the device is touched


def test_kernel_choice_by_shape():
    from wpt_b200 import ops
    assert ops.uses_stream(1, 32, 128) and ops.uses_stream(2, 32, 128) and ops.uses_stream(4, 16, 128)
    assert not ops.uses_stream(3, 32, 128)  # 96 columns: the prefill kernel
    assert not ops.uses_stream(1, 32, 64)   # head width 64: the prefill kernel
    assert ops._stream_shape(1, 32, False) == (32, 1)
    assert ops._stream_shape(3, 12, False) == (64, 5)
    assert ops._stream_shape(7, 12, True) == (16, 1)
    # key-stream plans (chunk tiles, splits, cluster) at the benchmarked decode shapes on 148 SMs
    assert ops._stream_plan_for(64, 1, 32, 32768, 0, 1024, False, 148, None) == (4, 2, True)   # window rows
    assert ops._stream_plan_for(64, 1, 32, 32768, 0, 0, False, 148, None) == (64, 4, False)    # two waves: merge
    assert ops._stream_plan_for(64, 1, 32, 32768, 1024, 1024, True, 148, None) == (8, 2, True)  # sparse gather
    assert ops._stream_plan_for(1, 1, 32, 262144, 0, 0, False, 148, None)[2] is False


def test_cluster_mode_takes_at_most_8_splits(library):
    # part_o == part_lse == NULL selects the in-cluster merge, which holds at most 8 splits
    from wpt_b200 import _lib
    lib = _lib.lib()
    rc = lib.wpt_attn_decode(None, None, None, 0, 0, 0, 0, None, None, None, 0, None, None, None, None, None, 9, 1,
                             1, 1, 32, 128, 1024, 0, 1.0, None)
    assert rc == _lib.ERR_INVALID and b"at most 8" in lib.wpt_last_error()


def test_prefill_without_scratch_takes_only_two_splits(library):
    # part_o == part_lse == NULL with 2 splits selects the prefill kernel's cluster combine; other split
    # counts need the scratch
    from wpt_b200 import _lib
    lib = _lib.lib()
    rc = lib.wpt_attn_prefill(None, None, None, 0, 0, 0, 0, None, None, None, None, None, None, None, None, None, 3,
                              1, 256, 16, 128, 1024, 0, 1.0, None)
    assert rc == _lib.ERR_INVALID and b"or neither, for 2" in lib.wpt_last_error()


def test_cpu_tensors_are_refused_not_computed():
    import wpt_b200
    q = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA device only"):
        wpt_b200.exact_attention(q, k, k, torch.arange(4), 0.1, 0, 2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_inputs_not_in_bfloat16_are_refused_not_rounded(dtype):
    # the reference computes in its inputs' dtype; rounding float32 inputs to
    # bf16 would return float32 tensors of bf16 accuracy, so they are refused
    # with the error the reference's kernel tests skip on
    import wpt_b200
    q = torch.zeros(1, 4, 2, 128, dtype=dtype)
    k = torch.zeros(1, 4, 128, dtype=dtype)
    sink = torch.zeros(2)
    empty = torch.zeros(1, 4, 0, dtype=torch.int64)
    calls = [lambda: wpt_b200.exact_attention(q, k, k, torch.arange(4), 0.1, 0, 2),
             lambda: wpt_b200.sparse_attention(q, k, k, sink, empty, torch.arange(4), 0.1, 2),
             lambda: wpt_b200.window_attention(q, k, k, sink, torch.arange(4), 0.1, window=1),
             lambda: wpt_b200.tree_attention(q, k, k, torch.tensor([0]), torch.arange(4) - 1, 0.1),
             lambda: wpt_b200.forward_with_lse(q, k, k, torch.arange(4), 0.1)]
    for call in calls:
        with pytest.raises(NotImplementedError, match="bfloat16"):
            call()


def test_module_has_the_reference_contract():
    import inspect

    import wpt_b200
    assert isinstance(wpt_b200.NAME, str)
    assert list(inspect.signature(wpt_b200.exact_attention).parameters) == [
        "q", "k", "v", "positions", "scale", "top_k", "window"]
    assert list(inspect.signature(wpt_b200.sparse_attention).parameters) == [
        "q", "k", "v", "sink", "idx", "positions", "scale", "window"]
    assert list(inspect.signature(wpt_b200.window_attention).parameters)[:6] == [
        "q", "k", "v", "sink", "positions", "scale"]
