"""Which kernel each kind of element-wise call launches.  Every path of
tadma_b200_eltwise gives the same bits, so the parity tests cannot see a call
that lands on a slower path; this test names the kernel (recorded by
torch.profiler's CUDA activity trace) that config 2's call and the common
eager calls must reach."""
import pytest

import tadma_b200 as tb
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, Op, instr, make_tensor

pytestmark = pytest.mark.gpu


def kernels_of(fn):
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    if not names:
        pytest.skip("the profiler recorded no CUDA kernels on this box")
    return " ".join(names)


def rnd(shape, dt):
    import torch
    t = torch.empty(shape, dtype=dt, device="cuda")
    tb.fill(t, Dist.NORMAL, 0.0, 1.0, seed=0, stream_id=1)
    return t


def test_config2_reaches_the_row_affine_kernel():
    import torch
    x, bias = rnd((256, 8192), torch.bfloat16), rnd((8192,), torch.bfloat16)
    y = torch.empty_like(x)
    bview = make_tensor(bias.data_ptr(), DType.BF16, [256, 8192], [0, 1])
    prog = [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32),
            instr(Op.GELU, round_dtype=DType.F32)]
    names = kernels_of(lambda: tb.eltwise(y, [x, bview], prog, Compute.F32))
    assert "affine_rows_kernel" in names, names


@pytest.mark.parametrize("case,kernel", [("add", "typed1_kernel"), ("cast", "typed1_kernel"),
                                         ("gt", "typed_cmp_kernel"), ("where", "typed_where_kernel"),
                                         ("chain", "typed_kernel"), ("transpose", "transpose16_kernel"),
                                         ("transpose32", "transpose32_kernel"),
                                         ("gelu_add", "chain_narrow_kernel")])
def test_eager_calls_reach_their_typed_kernels(case, kernel):
    import torch
    a, b = rnd((512, 1024), torch.float16), rnd((512, 1024), torch.float16)
    out = torch.empty_like(a)
    if case == "add":
        fn = lambda: tb.eltwise(out, [a, b], [instr(Op.ADD, b=1, round_dtype=DType.F16)])  # noqa: E731
    elif case == "cast":
        o32 = torch.empty((512, 1024), dtype=torch.float32, device="cuda")
        fn = lambda: tb.eltwise(o32, [a], [instr(Op.COPY)])  # noqa: E731
    elif case == "gt":
        ob = torch.empty((512, 1024), dtype=torch.bool, device="cuda")
        fn = lambda: tb.eltwise(ob, [a, b], [instr(Op.GT, b=1, round_dtype=DType.BOOL)])  # noqa: E731
    elif case == "where":
        c = a > b
        fn = lambda: tb.eltwise(out, [c, a, b], [instr(Op.WHERE, b=1, c=2)])  # noqa: E731
    elif case == "chain":
        fn = lambda: tb.eltwise(out, [a, b], [instr(Op.MUL, b=1), instr(Op.EXP), instr(Op.SUB, b=1)])  # noqa: E731
    elif case == "transpose":
        at = torch.empty((1024, 512), dtype=torch.float16, device="cuda")
        fn = lambda: tb.eltwise(at, [a.t()], [instr(Op.COPY)])  # noqa: E731
    elif case == "transpose32":
        a32 = torch.empty((512, 1024), dtype=torch.float32, device="cuda")
        at32 = torch.empty((1024, 512), dtype=torch.float32, device="cuda")
        fn = lambda: tb.eltwise(at32, [a32.t()], [instr(Op.COPY)])  # noqa: E731
    else:  # act(x * s + y): compile-time affine program
        fn = lambda: tb.eltwise(out, [a, b], [instr(Op.MUL, b=SRC_IMM, imm=0.5), instr(Op.ADD, b=1),  # noqa: E731
                                              instr(Op.GELU)])
    names = kernels_of(fn)
    assert kernel in names, names
