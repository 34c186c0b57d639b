"""ql_lora_colsum_noalloc (partials in the library's static device scratch) against
ql_lora_colsum (partials in a caller workspace), both through the C ABI on the GPU. Collected
last so that it also runs after every other GPU test has used the library."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _colsum(name, X, Y, scale, transpose, workspace=None):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib, ops

    n, ncols = X.shape
    R = Y.shape[1]
    out = torch.full((R, ncols) if transpose else (ncols, R), float("nan"), device=DEV)
    args = [X.data_ptr(), X.stride(0), ops.dtype_code(X.dtype), Y.data_ptr(),
            ops.dtype_code(Y.dtype), n, ncols, R, float(scale), int(transpose), out.data_ptr()]
    if workspace is not None:
        args += [workspace.data_ptr(), workspace.numel()]
    _lib.call(name, *args, torch.cuda.current_stream().cuda_stream)
    return out


@pytest.mark.parametrize("n,ncols,xdt,ydt,transpose", [
    (1090, 1536, torch.float16, torch.float16, False),
    (1090, 1536, torch.float16, torch.float32, True),
    (300, 8960, torch.bfloat16, torch.bfloat16, False),
    (37, 256, torch.bfloat16, torch.float32, True),
    (0, 64, torch.float16, torch.float16, False),
])
def test_noalloc_matches_workspace_entry_point(n, ncols, xdt, ydt, transpose):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib, ops

    g = torch.Generator(device=DEV).manual_seed(n * 13 + ncols)
    X = torch.randn(n, ncols, device=DEV, generator=g).to(xdt)
    Y = torch.randn(n, 16, device=DEV, generator=g).to(ydt)
    need = int(_lib.lib().ql_lora_colsum_workspace(n, ncols, 16))
    ws = torch.empty(max(need, 1), device=DEV, dtype=torch.float32)
    ref = _colsum("ql_lora_colsum", X, Y, 0.5, transpose, ws)
    first = _colsum("ql_lora_colsum_noalloc", X, Y, 0.5, transpose)
    second = _colsum("ql_lora_colsum_noalloc", X, Y, 0.5, transpose)  # scratch reused as left
    torch.cuda.synchronize()
    for got in (first, second):
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
    expect = 0.5 * (X.float().t() @ Y.float())
    if transpose:
        expect = expect.t()
    torch.testing.assert_close(first, expect, rtol=1e-3, atol=1e-3)
    assert ops.device_status() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib

    n, ncols = 1, 73728  # one split of 73,728 x 16 partials > 1,048,576 floats
    assert _lib.lib().ql_lora_colsum_workspace(n, ncols, 16) > 1048576
    X = torch.zeros(n, ncols, device=DEV, dtype=torch.float16)
    Y = torch.zeros(n, 16, device=DEV, dtype=torch.float16)
    with pytest.raises(_lib.QLError, match="floats of scratch"):
        _colsum("ql_lora_colsum_noalloc", X, Y, 1.0, False)


def test_noalloc_accepts_a_shape_that_fills_its_scratch_exactly():
    """One split of 65,536 columns x rank 16 needs exactly the 1,048,576 floats of the scratch:
    accepted, and equal to the workspace entry point's result (twice in a row)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib

    n, ncols = 1, 65536
    assert _lib.lib().ql_lora_colsum_workspace(n, ncols, 16) == 1048576
    g = torch.Generator(device=DEV).manual_seed(3)
    X = torch.randn(n, ncols, device=DEV, generator=g).half()
    Y = torch.randn(n, 16, device=DEV, generator=g).half()
    ws = torch.empty(1048576, device=DEV, dtype=torch.float32)
    ref = _colsum("ql_lora_colsum", X, Y, 1.0, False, ws)
    for _ in range(2):
        got = _colsum("ql_lora_colsum_noalloc", X, Y, 1.0, False)
        torch.cuda.synchronize()
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_bad_layouts_and_ranks():
    """Column counts that are not whole 8-column groups, and ranks other than 16, are refused
    with a status (BAD_ARG, UNSUPPORTED) before anything launches."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib, ops

    lib = _lib.lib()
    X = torch.zeros(4, 104, device=DEV, dtype=torch.float16)  # rows of 104, 100 of them used
    Y = torch.zeros(4, 16, device=DEV, dtype=torch.float16)
    out = torch.zeros(100, 16, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ql_lora_colsum_noalloc(X.data_ptr(), 104, ops.dtype_code(X.dtype), Y.data_ptr(),
                                    ops.dtype_code(Y.dtype), 4, 100, 16, 1.0, 0, out.data_ptr(),
                                    stream)
    assert rc == 1  # QL_STATUS_BAD_ARG: 100 columns are not whole 8-column groups
    rc = lib.ql_lora_colsum_noalloc(X.data_ptr(), 104, ops.dtype_code(X.dtype), Y.data_ptr(),
                                    ops.dtype_code(Y.dtype), 4, 96, 8, 1.0, 0, out.data_ptr(),
                                    stream)
    assert rc == 3 and b"rank 8" in lib.ql_last_error()  # QL_STATUS_UNSUPPORTED
