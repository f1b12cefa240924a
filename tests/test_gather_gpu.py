"""Gather (+ fused broadcast add) vs the oracle: bit-exact (index work plus one
fp32 add rounded once), error word for out-of-range ids."""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import Dist, DType, make_tensor
from tests.helpers import dev_view, empty_dev, from_dev, gen, to_dev

pytestmark = pytest.mark.gpu


def run_both(table, tdt, axis, ids, add, adt, out_dt):
    td = to_dev(table, tdt)
    idd = to_dev(ids)
    keep, ad = dev_view(add, adt) if add is not None else (None, None)
    oshape = list(table.shape[:axis]) + list(ids.shape) + list(table.shape[axis + 1:])
    out = empty_dev(oshape, out_dt)
    tb.gather(td, axis, idd, out, add=ad)
    flags = tb.error_flags(clear=True)
    ref = np.zeros(oshape, dtype=from_dev(out).dtype)
    rc = O.gather(table, axis, ids, ref, add, table_dtype=tdt, add_dtype=adt, out_dtype=out_dt)
    return from_dev(out), ref, flags, rc


def test_config5_small():
    # Config 5 at reduced size: fp16 table, int64 ids, bf16 pos broadcast over batch, bf16 out.
    V, B, S, D = 1000, 4, 64, 256
    table = gen((V, D), DType.F16, Dist.NORMAL, 0.0, 0.02, 1)
    ids = gen((B, S), DType.I64, Dist.INDEX, 0, V, 2)
    pos = gen((S, D), DType.BF16, Dist.NORMAL, 0.0, 0.02, 3)
    got, ref, flags, rc = run_both(table, DType.F16, 0, ids, np.broadcast_to(pos, (B, S, D)), DType.BF16, DType.BF16)
    assert rc == 0 and flags == 0
    assert np.array_equal(got, ref)
    ref2 = np.zeros_like(ref)
    O.lib().or_cfg5_gather_add(O.ptr(table), V, O.ptr(ids), O.ptr(pos), O.ptr(ref2), B, S, D)
    assert np.array_equal(ref2, ref)


def test_identity_table_kat():
    # KAT: gathering from an identity-like table returns the ids' rows.
    V = 64
    table = np.eye(V, dtype=np.float32)
    ids = np.array([[3, 0, 63], [5, 5, 1]], dtype=np.int64)
    got, ref, flags, rc = run_both(table, DType.F32, 0, ids, None, None, DType.F32)
    assert np.array_equal(got, np.eye(V, dtype=np.float32)[ids]) and np.array_equal(ref, got)


def test_negative_and_out_of_range_ids():
    V, D = 100, 64
    table = gen((V, D), DType.F32, Dist.NORMAL, 0, 1, 4)
    ids = np.array([[-1, 0, 99, -100]], dtype=np.int64)
    got, ref, flags, rc = run_both(table, DType.F32, 0, ids, None, None, DType.F32)
    assert flags == 0 and rc == 0
    assert np.array_equal(got[0], table[[99, 0, 99, 0]])
    ids = np.array([[1, 100, -101, 2]], dtype=np.int64)
    got, ref, flags, rc = run_both(table, DType.F32, 0, ids, None, None, DType.F32)
    assert flags & (1 << 4) and rc == 4
    assert np.all(got[0, 1] == 0) and np.all(got[0, 2] == 0)
    assert np.array_equal(got, ref)
    assert tb.error_flags() == 0  # cleared by the previous read


@pytest.mark.parametrize("tdt,adt,odt", [(DType.F32, DType.F32, DType.F32), (DType.BF16, DType.F16, DType.F32),
                                         (DType.F16, None, DType.F16)])
def test_dtype_combos_int32_ids(tdt, adt, odt):
    V, D = 300, 72
    table = gen((V, D), tdt, Dist.NORMAL, 0, 1, 5)
    ids = gen((3, 5, 7), DType.I32, Dist.INDEX, 0, V, 6)
    add = gen((1, 5, 1, ), adt, Dist.NORMAL, 0, 1, 7) if adt is not None else None
    addv = np.broadcast_to(add[..., None], (3, 5, 7, D)) if add is not None else None
    got, ref, flags, rc = run_both(table, tdt, 0, ids, addv, adt, odt)
    assert rc == 0 and np.array_equal(got, ref)


def test_generic_path_axis1_odd_width():
    table = gen((6, 50, 5), DType.F32, Dist.NORMAL, 0, 1, 8)
    ids = np.array([[0, 49], [7, 3]], dtype=np.int64)
    got, ref, flags, rc = run_both(table, DType.F32, 1, ids, None, None, DType.F32)
    assert rc == 0 and np.array_equal(got, ref)
    assert np.array_equal(got, table[:, ids, :])


def test_config5_full_size_sampled():
    # Full config 5 at one GPU: table [50257, 4096] fp16, ids [2048, 4096] int64,
    # pos [4096, 4096] bf16 -> out [2048, 4096, 4096] bf16 (68.7 GB).
    import torch
    V, B, S, D = 50257, 2048, 4096, 4096
    table = empty_dev((V, D), DType.F16)
    ids = empty_dev((B, S), DType.I64)
    pos = empty_dev((S, D), DType.BF16)
    tb.fill(table, Dist.NORMAL, 0.0, 0.02, 0, 1)
    tb.fill(ids, Dist.INDEX, 0, V, 0, 2)
    tb.fill(pos, Dist.NORMAL, 0.0, 0.02, 0, 3)
    out = empty_dev((B, S, D), DType.BF16)
    tb.gather(table, 0, ids, out, add=make_tensor(pos.data_ptr(), DType.BF16, [B, S, D], [0, D, 1]))
    assert tb.error_flags() == 0
    rng = np.random.default_rng(3)
    bs, ss = rng.integers(0, B, 128), rng.integers(0, S, 128)
    got = from_dev(out[torch.as_tensor(bs, device="cuda"), torch.as_tensor(ss, device="cuda")])
    idh = from_dev(ids)[bs, ss]
    th = from_dev(table[torch.as_tensor(idh, device="cuda")])
    ph = from_dev(pos[torch.as_tensor(ss, device="cuda")])
    ref = np.zeros_like(got)
    rows = np.arange(128, dtype=np.int64)  # keep alive across the C call
    O.lib().or_cfg5_gather_add(O.ptr(th), 128, O.ptr(rows), O.ptr(ph), O.ptr(ref), 1, 128, D)
    assert np.array_equal(got, ref)
    del out
    torch.cuda.empty_cache()


# --- row path edges: row lengths that are not a multiple of a warp's 256-element
# step, fp32 operands, many rows per warp (the next id is loaded a row
# ahead), invalid ids mid-stream, strided ids, padded output rows.

@pytest.mark.parametrize("tdt,adt,odt,D", [(DType.F16, DType.BF16, DType.BF16, 1032),  # ragged last step
                                           (DType.F32, DType.F32, DType.F32, 520),
                                           (DType.BF16, None, DType.F32, 2056),        # no add
                                           (DType.F16, DType.F32, DType.F16, 64)])     # one short row
def test_row_lengths_and_dtypes(tdt, adt, odt, D):
    V, B, S = 777, 3, 37
    table = gen((V, D), tdt, Dist.NORMAL, 0, 1, 11)
    ids = gen((B, S), DType.I64, Dist.INDEX, 0, V, 12)
    add = np.broadcast_to(gen((S, D), adt, Dist.NORMAL, 0, 1, 13), (B, S, D)) if adt is not None else None
    got, ref, flags, rc = run_both(table, tdt, 0, ids, add, adt, odt)
    assert rc == 0 and flags == 0 and np.array_equal(got, ref)


def test_many_rows_with_invalid_ids():
    # 204800 rows: each warp walks tens of rows, loading each next id ahead.
    V, B, S, D = 5000, 400, 512, 64
    table = gen((V, D), DType.F16, Dist.NORMAL, 0, 1, 14)
    ids = gen((B, S), DType.I64, Dist.INDEX, 0, V, 15)
    ids[7, 100] = V          # out of range
    ids[399, 511] = -V - 1   # out of range, last row
    ids[200, 0] = -1         # valid (wraps to V-1)
    pos = gen((S, D), DType.BF16, Dist.NORMAL, 0, 1, 16)
    got, ref, flags, rc = run_both(table, DType.F16, 0, ids, np.broadcast_to(pos, (B, S, D)), DType.BF16, DType.BF16)
    assert rc == 4 and flags & (1 << 4)
    assert np.array_equal(got, ref)
    assert np.array_equal(got[7, 100], pos[100])  # table part zero, pos still added


def test_strided_ids_and_padded_out_rows():
    import torch
    V, R, D = 900, 300, 256
    table = gen((V, D), DType.F16, Dist.NORMAL, 0, 1, 17)
    ids_full = gen((R, 2), DType.I64, Dist.INDEX, 0, V, 18)
    idd = to_dev(ids_full)[:, 1]                      # stride 2 ids
    out_full = torch.zeros((R, D + 64), dtype=torch.float16, device="cuda")
    out = out_full[:, 8:8 + D]                        # padded rows, 16-byte aligned start
    tb.gather(to_dev(table), 0, idd, out)
    assert tb.error_flags(clear=True) == 0
    got = from_dev(out_full)
    assert np.array_equal(got[:, 8:8 + D], table[ids_full[:, 1]])
    assert not got[:, :8].any() and not got[:, 8 + D:].any()
