"""tadma_b200_row_program: decomposed normalisations (LayerNorm, softmax,
RMSNorm, a residual add before a LayerNorm) as one row pass give the bits of
the separate calls (tadma_b200_reduce, tadma_b200_reduce_chain_post,
tadma_b200_eltwise), stage outputs included; the LayerNorm also against the
oracle.  fp32, fp16 and bf16 rows."""
import numpy as np
import pytest
import torch

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, DType, LNMode, Op, Reduce, instr, make_tensor

pytestmark = pytest.mark.gpu

TDT = {DType.F32: torch.float32, DType.F16: torch.float16, DType.BF16: torch.bfloat16}


def _bits(t):
    t = t.contiguous().cpu()
    return t.view(torch.int32 if t.element_size() == 4 else torch.int16).numpy()


def _rows_view(t, rows, cols):
    return make_tensor(t.data_ptr(), tb.torch_dtype_code(t), [rows, cols], [cols, 1])


def _col_view(t, rows, cols):
    return make_tensor(t.data_ptr(), tb.torch_dtype_code(t), [rows, cols], [0, 1])


def _scalar_view(t, rows, cols):
    return make_tensor(t.data_ptr(), tb.torch_dtype_code(t), [rows, cols], [1, 0])


def _vec(t, rows):
    return make_tensor(t.data_ptr(), tb.torch_dtype_code(t), [rows], [1])


def _inputs(dt, rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(rows, cols, device="cuda", generator=g) * 2 + 0.5).to(TDT[dt])
    gamma = (1 + 0.1 * torch.randn(cols, device="cuda", generator=g)).to(TDT[dt])
    beta = (0.1 * torch.randn(cols, device="cuda", generator=g)).to(TDT[dt])
    return x, gamma, beta


def _edge_rows(x, dt):
    """Rows whose quotients leave the fused division's range: a constant row
    (every x - mean is zero), and for fp32 rows of magnitude 1e20 and 1e-20,
    a row holding an infinity and one holding a NaN."""
    x[0] = 0.5
    if dt == DType.F32 and x.shape[0] >= 6:
        x[1] *= 1e20
        x[2] *= 1e-20
        x[3, 7] = float("inf")
        x[4, 3] = float("nan")
        x[5, ::3] = 0.0


@pytest.mark.parametrize("dt", [DType.F32, DType.F16, DType.BF16])
@pytest.mark.parametrize("rows,cols,edges", [(300, 768, False), (37, 1024, False), (1, 64, False), (1000, 128, False),
                                             (64, 768, True), (40, 96, True)])
def test_layer_norm_decomposition_one_pass(dt, rows, cols, edges):
    if dt == DType.F32 and cols > 1024:
        pytest.skip("fp32 rows up to 1024")
    x, gamma, beta = _inputs(dt, rows, cols, rows + cols)
    if edges:
        _edge_rows(x, dt)
    eps = 1e-12
    sdt = TDT[dt]
    # separate calls, as deferred evaluation issues them
    m_sep = torch.empty(rows, 1, dtype=sdt, device="cuda")
    tb.reduce(Reduce.MEAN, x, -1, m_sep)
    sd_sep = torch.empty(rows, 1, dtype=sdt, device="cuda")
    post = [instr(Op.COPY, round_dtype=dt), instr(Op.ADD, b=SRC_IMM, imm=eps, round_dtype=dt),
            instr(Op.SQRT, round_dtype=dt)]
    tb.reduce_chain(Reduce.MEAN, [x, _scalar_view(m_sep, rows, cols)],
                    [instr(Op.SUB, b=1, round_dtype=dt), instr(Op.POW, b=SRC_IMM, imm=2.0, round_dtype=dt)], -1,
                    sd_sep, Compute.F32, post=post)
    y_sep = torch.empty_like(x)
    tail = [instr(Op.SUB, b=1, round_dtype=dt), instr(Op.DIV, b=2, round_dtype=dt), instr(Op.MUL, b=3, round_dtype=dt),
            instr(Op.ADD, b=4, round_dtype=dt)]
    tb.eltwise(y_sep, [x, _scalar_view(m_sep, rows, cols), _scalar_view(sd_sep, rows, cols),
                       _col_view(gamma, rows, cols), _col_view(beta, rows, cols)], tail, Compute.F32)
    # one row program: operands x, gamma, beta; stages m (3), sd (4)
    m = torch.empty(rows, dtype=sdt, device="cuda")
    sd = torch.empty(rows, dtype=sdt, device="cuda")
    y = torch.empty_like(x)
    stages = [
        (Reduce.MEAN, [], [], _vec(m, rows), 0),
        (Reduce.MEAN, [instr(Op.SUB, b=3, round_dtype=dt), instr(Op.POW, b=SRC_IMM, imm=2.0, round_dtype=dt)], post,
         _vec(sd, rows), 0),
    ]
    prog = [instr(Op.SUB, b=3, round_dtype=dt), instr(Op.DIV, b=4, round_dtype=dt), instr(Op.MUL, b=1, round_dtype=dt),
            instr(Op.ADD, b=2, round_dtype=dt)]
    tb.row_program(rows, cols, [_rows_view(x, rows, cols), _col_view(gamma, rows, cols), _col_view(beta, rows, cols)],
                   stages, prog, _rows_view(y, rows, cols))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(m), _bits(m_sep).reshape(-1))
    assert np.array_equal(_bits(sd), _bits(sd_sep).reshape(-1))
    assert np.array_equal(_bits(y), _bits(y_sep))
    if dt == DType.F32 and not edges:
        xn, gn, bn = x.cpu().numpy(), gamma.cpu().numpy(), beta.cpu().numpy()
        ref = np.zeros_like(xn)
        assert O.layer_norm(xn, -1, gn, bn, eps, LNMode.ONNX, ref) == 0
        assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * np.sqrt(cols) * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("dt", [DType.F32, DType.BF16])
def test_softmax_decomposition_one_pass(dt):
    rows, cols = 513, 512
    x, _, _ = _inputs(dt, rows, cols, 7)
    x[5, 17] = 40.0  # a large logit: max-subtraction matters
    sdt = TDT[dt]
    mx_sep = torch.empty(rows, 1, dtype=sdt, device="cuda")
    tb.reduce(Reduce.MAX, x, -1, mx_sep)
    den_sep = torch.empty(rows, 1, dtype=sdt, device="cuda")
    tb.reduce_chain(Reduce.SUM, [x, _scalar_view(mx_sep, rows, cols)],
                    [instr(Op.SUB, b=1, round_dtype=dt), instr(Op.EXP, round_dtype=dt)], -1, den_sep, Compute.F32)
    y_sep = torch.empty_like(x)
    tb.eltwise(y_sep, [x, _scalar_view(mx_sep, rows, cols), _scalar_view(den_sep, rows, cols)],
               [instr(Op.SUB, b=1, round_dtype=dt), instr(Op.EXP, round_dtype=dt), instr(Op.DIV, b=2, round_dtype=dt)])
    mx = torch.empty(rows, dtype=sdt, device="cuda")
    den = torch.empty(rows, dtype=sdt, device="cuda")
    y = torch.empty_like(x)
    tb.row_program(rows, cols, [_rows_view(x, rows, cols)],
                   [(Reduce.MAX, [], [], _vec(mx, rows), 0),
                    (Reduce.SUM, [instr(Op.SUB, b=1, round_dtype=dt), instr(Op.EXP, round_dtype=dt)], [], _vec(den, rows), 0)],
                   [instr(Op.SUB, b=1, round_dtype=dt), instr(Op.EXP, round_dtype=dt), instr(Op.DIV, b=2, round_dtype=dt)],
                   _rows_view(y, rows, cols))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(mx), _bits(mx_sep).reshape(-1))
    assert np.array_equal(_bits(den), _bits(den_sep).reshape(-1))
    assert np.array_equal(_bits(y), _bits(y_sep))
    ref = torch.softmax(x.float(), dim=-1)
    tol = 1e-6 if dt == DType.F32 else 2e-2  # bf16: each of the three steps rounds to 8 bits
    assert (y.float() - ref).abs().max().item() <= tol


def test_rms_norm_and_residual_two_row_operands():
    rows, cols, dt = 256, 1024, DType.F16
    x, gamma, beta = _inputs(dt, rows, cols, 11)
    r, _, _ = _inputs(dt, rows, cols, 12)
    sdt = TDT[dt]
    # h = x + r; rms = sqrt(mean(h^2) + eps); y = h / rms * gamma
    rms_sep = torch.empty(rows, 1, dtype=sdt, device="cuda")
    post = [instr(Op.COPY, round_dtype=dt), instr(Op.ADD, b=SRC_IMM, imm=1e-6, round_dtype=dt),
            instr(Op.SQRT, round_dtype=dt)]
    tb.reduce_chain(Reduce.MEAN, [x, r], [instr(Op.ADD, b=1, round_dtype=dt), instr(Op.POW, b=SRC_IMM, imm=2.0,
                                                                                      round_dtype=dt)],
                    -1, rms_sep, Compute.F32, post=post)
    y_sep = torch.empty_like(x)
    tb.eltwise(y_sep, [x, r, _scalar_view(rms_sep, rows, cols), _col_view(gamma, rows, cols)],
               [instr(Op.ADD, b=1, round_dtype=dt), instr(Op.DIV, b=2, round_dtype=dt), instr(Op.MUL, b=3, round_dtype=dt)])
    rms = torch.empty(rows, dtype=sdt, device="cuda")
    y = torch.empty_like(x)
    tb.row_program(rows, cols, [_rows_view(x, rows, cols), _rows_view(r, rows, cols), _col_view(gamma, rows, cols)],
                   [(Reduce.MEAN, [instr(Op.ADD, b=1, round_dtype=dt), instr(Op.POW, b=SRC_IMM, imm=2.0, round_dtype=dt)],
                     post, _vec(rms, rows), 0)],
                   [instr(Op.ADD, b=1, round_dtype=dt), instr(Op.DIV, b=3, round_dtype=dt), instr(Op.MUL, b=2, round_dtype=dt)],
                   _rows_view(y, rows, cols))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(rms), _bits(rms_sep).reshape(-1))
    assert np.array_equal(_bits(y), _bits(y_sep))


def test_unsupported_grids_launch_nothing():
    rows, cols = 4, 4096  # fp32 rows longer than 1024 values
    x = torch.zeros(rows, cols, device="cuda")
    y = torch.full_like(x, 3.0)
    m = torch.empty(rows, device="cuda")
    with pytest.raises(tb.TadmaError) as e:
        tb.row_program(rows, cols, [_rows_view(x, rows, cols)], [(Reduce.MEAN, [], [], _vec(m, rows), 0)],
                       [instr(Op.SUB, b=1)], _rows_view(y, rows, cols))
    assert e.value.code == tb.Status.ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert bool((y == 3.0).all())
