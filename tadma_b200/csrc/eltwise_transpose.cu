// eltwise_transpose.cu - chains over a transposed view: tiled transposes
// through shared memory.
#include "eltwise_impl.cuh"

namespace tadma_b200 {
namespace {

// ---------------------------------------------------------- tiled transpose --
// One input whose unit-stride dim is not the output's: a copy through a
// transpose (contiguous() after transpose<0,2,3,1>, a cast of a transposed
// view).  Element-at-a-time, one side of the copy would be uncoalesced; here
// a CTA stages a 32 x 32 tile in shared memory, reading along the input's
// contiguous dim and writing along the output's, and runs the chain on each
// element on the way out.  Remaining dims are batch dims (grid z).

template <int PROG>
__global__ void __launch_bounds__(THREADS) transpose_chain_kernel(const __grid_constant__ TransposeParams tp) {
    pdl_begin();
    __shared__ float tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    const int64_t i0 = (int64_t)blockIdx.y * 32, j0 = (int64_t)blockIdx.x * 32;
    for (int64_t bz = blockIdx.z; bz < tp.nbatch; bz += gridDim.z) {
        uint64_t e = (uint64_t)bz;
        int64_t ib = 0, ob = 0;
        for (int d = tp.nb - 1; d >= 1; d--) {
            uint64_t q, r;
            tp.bdm[d].divmod(e, q, r);
            ib += (int64_t)r * tp.b_in[d];
            ob += (int64_t)r * tp.b_out[d];
            e = q;
        }
        if (tp.nb > 0) {
            ib += (int64_t)e * tp.b_in[0];
            ob += (int64_t)e * tp.b_out[0];
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t i = i0 + tx, j = j0 + ty + 8 * k;
            if (i < tp.n_i && j < tp.n_j) tile[ty + 8 * k][tx] = load_as<float>(tp.in, tp.in_dtype, ib + i + j * tp.in_sj);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t i = i0 + ty + 8 * k, j = j0 + tx;
            if (i < tp.n_i && j < tp.n_j) {
                float val[1][1] = {{tile[tx][ty + 8 * k]}};
                float acc[1] = {val[0][0]};
                program<float, 1, 1, PROG>(tp.chain, acc, val);
                store_from(tp.out, tp.out_dtype, ob + i * tp.out_si + j, acc[0]);
            }
        }
        __syncthreads();
    }
}

// 64 x 64 tiles with 16-byte accesses on both sides, for f32 / f16 / bf16 in
// and out with 16-byte aligned rows and fp32 on at least one side (16-bit in
// and out goes to transpose16_kernel): each thread loads 2 (16-bit) or 4 (f32)
// 16-byte vectors along the input's contiguous dim, the tile is transposed
// through shared memory as fp32, and each thread stores 2 vectors of 8
// elements along the output's contiguous dim.  One tile per CTA.  The 32 x 32
// element-at-a-time kernel above (the fallback for other layouts) kept too
// few bytes in flight: ~1.0 TB/s for a 16-bit transpose.
template <typename TI, typename TO, int PROG>
__global__ void __launch_bounds__(THREADS) transpose64_kernel(const __grid_constant__ TransposeParams tp) {
    pdl_begin();
    constexpr int T = 64;
    constexpr int VI = 16 / (int)sizeof(TI);        // input elements per 16-byte load
    constexpr int LV = T * (T / VI) / THREADS;       // loads per thread
    constexpr int SV = T * (T / 8) / THREADS;        // 8-element stores per thread
    __shared__ float tile[T][T + 1];                 // [j][i]
    const int64_t i0 = (int64_t)blockIdx.y * T, j0 = (int64_t)blockIdx.x * T;
    for (int64_t bz = blockIdx.z; bz < tp.nbatch; bz += gridDim.z) {
        uint64_t e = (uint64_t)bz;
        int64_t ib = 0, ob = 0;
        for (int d = tp.nb - 1; d >= 1; d--) {
            uint64_t q, r;
            tp.bdm[d].divmod(e, q, r);
            ib += (int64_t)r * tp.b_in[d];
            ob += (int64_t)r * tp.b_out[d];
            e = q;
        }
        if (tp.nb > 0) {
            ib += (int64_t)e * tp.b_in[0];
            ob += (int64_t)e * tp.b_out[0];
        }
        const TI* in = reinterpret_cast<const TI*>(tp.in) + ib;
        uint4 r[LV];
#pragma unroll
        for (int u = 0; u < LV; u++) {
            const int q = threadIdx.x + THREADS * u;
            const int jj = q / (T / VI), ii = (q % (T / VI)) * VI;
            const int64_t i = i0 + ii, j = j0 + jj;
            if (i < tp.n_i && j < tp.n_j) r[u] = ld_stream_v4(in + i + j * tp.in_sj);
        }
#pragma unroll
        for (int u = 0; u < LV; u++) {
            const int q = threadIdx.x + THREADS * u;
            const int jj = q / (T / VI), ii = (q % (T / VI)) * VI;
            if (i0 + ii < tp.n_i && j0 + jj < tp.n_j) {
                float f[8];
                if constexpr (sizeof(TI) == 4) {
                    f[0] = __uint_as_float(r[u].x);
                    f[1] = __uint_as_float(r[u].y);
                    f[2] = __uint_as_float(r[u].z);
                    f[3] = __uint_as_float(r[u].w);
                } else {
                    unpack8(r[u], std::is_same<TI, __half>::value ? TADMA_F16 : TADMA_BF16, f);
                }
#pragma unroll
                for (int k = 0; k < VI; k++) tile[jj][ii + k] = f[k];
            }
        }
        __syncthreads();
        TO* out = reinterpret_cast<TO*>(tp.out) + ob;
#pragma unroll
        for (int u = 0; u < SV; u++) {
            const int q = threadIdx.x + THREADS * u;
            const int ii = q >> 3, jj = (q & 7) * 8;
            const int64_t i = i0 + ii, j = j0 + jj;
            if (i < tp.n_i && j < tp.n_j) {
                float val[1][8], acc[8];
#pragma unroll
                for (int k = 0; k < 8; k++) acc[k] = val[0][k] = tile[jj + k][ii];
                program<float, 1, 8, PROG>(tp.chain, acc, val);
                raw8_store<TO>(out + i * tp.out_si + j, acc);
            }
        }
        __syncthreads();
    }
}

// 16-bit in and out: 64 (i) x TJ (j) tiles kept as 16-bit element pairs.
// Each thread loads the same 16-byte chunk (8 values of i) from two adjacent
// input rows j, j + 1 and packs value k of both into one 32-bit word: the
// output row i + k's elements j, j + 1.  Words go to shared memory as
// W[i][j / 2]; the output side reads 16-byte chunks of 4 words (8 values of
// j) and stores them along the output's contiguous dim.  The 4-word chunks of
// row i are swizzled by XOR with (i / 8) % 8, so the scalar word stores (8
// rows i = 8c + k, c = 0..7, per warp) and the 16-byte reads (8 consecutive
// chunks per quarter warp) each cover all 32 banks once.  Half the shared
// memory traffic of an fp32 tile, and TJ = 256 keeps 32 KB of loads in flight
// per CTA (4x the 64 x 64 tile).  RAW: the chain is an identity on the same
// dtype, so words are stored untouched (bit-exact, NaN payloads included).
template <typename TI, typename TO, int PROG, int TJ, bool RAW>
__global__ void __launch_bounds__(THREADS, 4) transpose16_kernel(const __grid_constant__ TransposeParams tp) {
    pdl_begin();
    static_assert(sizeof(TI) == 2 && sizeof(TO) == 2 && (TJ == 128 || TJ == 256));
    constexpr int TI_ = 64;
    constexpr int WPR = TJ / 2;                  // words per W row
    constexpr int NP = TJ / 64;                  // row pairs per thread (32 pairs per pass)
    constexpr int CPR = TJ / 8;                  // 16-byte output chunks per W row
    constexpr int RPP = THREADS / CPR;           // W rows per output pass
    constexpr int NS = TI_ / RPP;                // output chunks per thread
    __shared__ __align__(16) uint32_t W[TI_ * WPR];
    const int t = threadIdx.x;
    const int c = t & 7, p0 = t >> 3;            // input chunk (i = 8c..8c+7), first row pair
    const int q = t % CPR, r0 = t / CPR;         // output chunk (j = 8q..8q+7), first W row
    const int64_t i0 = (int64_t)blockIdx.y * TI_, j0 = (int64_t)blockIdx.x * TJ;
    for (int64_t bz = blockIdx.z; bz < tp.nbatch; bz += gridDim.z) {
        uint64_t e = (uint64_t)bz;
        int64_t ib = 0, ob = 0;
        for (int d = tp.nb - 1; d >= 1; d--) {
            uint64_t qq, rr;
            tp.bdm[d].divmod(e, qq, rr);
            ib += (int64_t)rr * tp.b_in[d];
            ob += (int64_t)rr * tp.b_out[d];
            e = qq;
        }
        if (tp.nb > 0) {
            ib += (int64_t)e * tp.b_in[0];
            ob += (int64_t)e * tp.b_out[0];
        }
        const TI* in = reinterpret_cast<const TI*>(tp.in) + ib;
        const int64_t i = i0 + 8 * c;
        uint4 a[NP], b[NP];
#pragma unroll
        for (int u = 0; u < NP; u++) {
            const int64_t j = j0 + 2 * (p0 + 32 * u);
            // n_j is a multiple of 8, so j < n_j implies j + 1 < n_j.
            if (i < tp.n_i && j < tp.n_j) {
                a[u] = ld_stream_v4(in + i + j * tp.in_sj);
                b[u] = ld_stream_v4(in + i + (j + 1) * tp.in_sj);
            } else {
                a[u] = b[u] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < NP; u++) {
            const int p = p0 + 32 * u;
            const int pw = (((p >> 2) ^ c) << 2) | (p & 3);  // swizzled word of row 8c + k
            const uint32_t av[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
            const uint32_t bv[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
            for (int h = 0; h < 4; h++) {
                W[(8 * c + 2 * h) * WPR + pw] = __byte_perm(av[h], bv[h], 0x5410);
                W[(8 * c + 2 * h + 1) * WPR + pw] = __byte_perm(av[h], bv[h], 0x7632);
            }
        }
        __syncthreads();
        TO* out = reinterpret_cast<TO*>(tp.out) + ob;
#pragma unroll
        for (int u = 0; u < NS; u++) {
            const int row = r0 + RPP * u;
            const int64_t oi = i0 + row, oj = j0 + 8 * q;
            if (oi < tp.n_i && oj < tp.n_j) {
                const uint4 w = *reinterpret_cast<const uint4*>(&W[row * WPR + ((q ^ ((row >> 3) & 7)) << 2)]);
                if constexpr (RAW) {
                    st_stream_v4(out + oi * tp.out_si + oj, w);
                } else {
                    float val[1][8], acc[8];
                    unpack8(w, std::is_same<TI, __half>::value ? TADMA_F16 : TADMA_BF16, val[0]);
#pragma unroll
                    for (int k = 0; k < 8; k++) acc[k] = val[0][k];
                    program<float, 1, 8, PROG>(tp.chain, acc, val);
                    raw8_store<TO>(out + oi * tp.out_si + oj, acc);
                }
            }
        }
        __syncthreads();
    }
}

bool identity_chain(const TransposeParams& tp);

// fp32 in: 64 (i) x TJ (j) tiles of 32-bit words, W[i][j].  A warp loads
// 4 input rows j x 8 consecutive 16-byte chunks of i (four 128-byte runs)
// and stores each chunk's 4 values as scalar words down rows 4c .. 4c + 3
// of W; the output side reads 16-byte chunks of 4 words (4 values of j) and
// stores them along the output's contiguous dim, one W row per warp.  The
// 4-word chunks of row i sit XOR-swizzled by (i / 4) % 8, so the scalar
// stores (8 chunks c x 4 rows j per warp) and the 16-byte reads (8
// consecutive chunks per quarter warp) each cover the 32 banks once; the
// 64 x 64 fp32 tile of transpose64_kernel, padded rather than swizzled, read
// its words one at a time with 2-way conflicts.  TJ = 128 keeps 32 KB of
// loads in flight per CTA.  RAW: an identity chain copies the words.
template <typename TO, int PROG, int TJ, bool RAW>
__global__ void __launch_bounds__(THREADS, 4) transpose32_kernel(const __grid_constant__ TransposeParams tp) {
    pdl_begin();
    static_assert(TJ == 64 || TJ == 128);
    constexpr int TI_ = 64;
    constexpr int NL = (TJ / 4) * 2 / (THREADS / 32);  // load tasks (4 rows x 8 chunks) per warp
    constexpr int CPR = TJ / 4;                        // 16-byte output chunks per W row
    constexpr int RPP = THREADS / CPR;                 // W rows per output pass
    constexpr int NS = TI_ / RPP;                      // output chunks per thread
    __shared__ __align__(16) uint32_t W[TI_ * TJ];
    const int t = threadIdx.x, w = t >> 5, lane = t & 31;
    const int jl = lane & 3, cl = lane >> 2;  // load: row j within the 4, chunk within the 8
    const int q = t % CPR, r0 = t / CPR;      // output chunk (j = 4q .. 4q + 3), first W row
    const int64_t i0 = (int64_t)blockIdx.y * TI_, j0 = (int64_t)blockIdx.x * TJ;
    for (int64_t bz = blockIdx.z; bz < tp.nbatch; bz += gridDim.z) {
        uint64_t e = (uint64_t)bz;
        int64_t ib = 0, ob = 0;
        for (int d = tp.nb - 1; d >= 1; d--) {
            uint64_t qq, rr;
            tp.bdm[d].divmod(e, qq, rr);
            ib += (int64_t)rr * tp.b_in[d];
            ob += (int64_t)rr * tp.b_out[d];
            e = qq;
        }
        if (tp.nb > 0) {
            ib += (int64_t)e * tp.b_in[0];
            ob += (int64_t)e * tp.b_out[0];
        }
        const float* in = reinterpret_cast<const float*>(tp.in) + ib;
        uint4 a[NL];
#pragma unroll
        for (int u = 0; u < NL; u++) {
            const int k = w + (THREADS / 32) * u;  // task: rows 4 (k >> 1) .., chunks 8 (k & 1) ..
            const int c = 8 * (k & 1) + cl;
            const int64_t i = i0 + 4 * c, j = j0 + 4 * (k >> 1) + jl;
            a[u] = (i < tp.n_i && j < tp.n_j) ? ld_stream_v4(in + i + j * tp.in_sj) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < NL; u++) {
            const int k = w + (THREADS / 32) * u;
            const int c = 8 * (k & 1) + cl;
            const int cj = k >> 1;                                // 4-word chunk of j in W's rows
            const int col = ((cj ^ (c & 7)) << 2) | jl;           // swizzled word of rows 4c .. 4c + 3
            const uint32_t av[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
#pragma unroll
            for (int h = 0; h < 4; h++) W[(4 * c + h) * TJ + col] = av[h];
        }
        __syncthreads();
        TO* out = reinterpret_cast<TO*>(tp.out) + ob;
#pragma unroll
        for (int u = 0; u < NS; u++) {
            const int row = r0 + RPP * u;
            const int64_t oi = i0 + row, oj = j0 + 4 * q;
            if (oi < tp.n_i && oj < tp.n_j) {
                const uint4 v = *reinterpret_cast<const uint4*>(&W[row * TJ + ((q ^ ((row >> 2) & 7)) << 2)]);
                if constexpr (RAW) {
                    st_stream_v4(out + oi * tp.out_si + oj, v);
                } else {
                    float val[1][4] = {{__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w)}};
                    float acc[4] = {val[0][0], val[0][1], val[0][2], val[0][3]};
                    program<float, 1, 4, PROG>(tp.chain, acc, val);
                    if constexpr (sizeof(TO) == 4) {
                        st_stream_v4(out + oi * tp.out_si + oj, make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]),
                                                                           __float_as_uint(acc[2]), __float_as_uint(acc[3])));
                    } else {
                        const float f8[8] = {acc[0], acc[1], acc[2], acc[3], 0.0f, 0.0f, 0.0f, 0.0f};
                        const uint4 p = pack8(f8, std::is_same<TO, __half>::value ? TADMA_F16 : TADMA_BF16);
                        __stcs(reinterpret_cast<uint2*>(out + oi * tp.out_si + oj), make_uint2(p.x, p.y));
                    }
                }
            }
        }
        __syncthreads();
    }
}

template <typename TO, int TJ>
void launch_t32_tj(bool fast, dim3 grid, const TransposeParams& tp, cudaStream_t s) {
    if (identity_chain(tp)) (void)launch_pdl(transpose32_kernel<TO, PROG_INTERP, TJ, true>, grid, dim3(THREADS), 0, s, tp);
    else if (fast && sizeof(TO) == 2) (void)launch_pdl(transpose32_kernel<TO, PROG_INTERP_FAST, TJ, false>, grid, dim3(THREADS), 0, s, tp);
    else (void)launch_pdl(transpose32_kernel<TO, PROG_INTERP, TJ, false>, grid, dim3(THREADS), 0, s, tp);
}
template <typename TO>
void launch_t32_o(bool fast, int64_t gz, const TransposeParams& tp, cudaStream_t s) {
    const unsigned gy = (unsigned)((tp.n_i + 63) / 64);
    if (tp.n_j >= 128) launch_t32_tj<TO, 128>(fast, dim3((unsigned)((tp.n_j + 127) / 128), gy, (unsigned)gz), tp, s);
    else launch_t32_tj<TO, 64>(fast, dim3((unsigned)((tp.n_j + 63) / 64), gy, (unsigned)gz), tp, s);
}

template <typename TI, typename TO>
void launch_t64_io(bool fast, dim3 grid, const TransposeParams& tp, cudaStream_t s) {
    if (fast && sizeof(TO) == 2) (void)launch_pdl(transpose64_kernel<TI, TO, PROG_INTERP_FAST>, grid, dim3(THREADS), 0, s, tp);
    else (void)launch_pdl(transpose64_kernel<TI, TO, PROG_INTERP>, grid, dim3(THREADS), 0, s, tp);
}
template <typename TI>
void launch_t64_i(bool fast, dim3 grid, const TransposeParams& tp, cudaStream_t s) {
    switch (tp.out_dtype) {
    case TADMA_F32: launch_t64_io<TI, float>(fast, grid, tp, s); break;
    case TADMA_F16: launch_t64_io<TI, __half>(fast, grid, tp, s); break;
    default: launch_t64_io<TI, __nv_bfloat16>(fast, grid, tp, s); break;
    }
}

// Whether transpose64_kernel covers this layout: f32 / f16 / bf16 on both
// sides, every row start and batch offset 16-byte aligned, and whole vectors
// at the edges (n_i a multiple of the input vector, n_j of 8).
bool transpose64_ok(const TransposeParams& tp) {
    auto fdt = [](int dt) { return dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16; };
    if (!fdt(tp.in_dtype) || !fdt(tp.out_dtype)) return false;
    const int64_t ei = dtype_size(tp.in_dtype), eo = dtype_size(tp.out_dtype);
    if ((uintptr_t)tp.in % 16 || (uintptr_t)tp.out % 16) return false;
    if ((tp.in_sj * ei) % 16 || (tp.out_si * eo) % 16) return false;
    for (int d = 0; d < tp.nb; d++)
        if ((tp.b_in[d] * ei) % 16 || (tp.b_out[d] * eo) % 16) return false;
    if (tp.n_i % (16 / ei) || tp.n_j % 8) return false;
    return (tp.n_i + 63) / 64 <= 65535;
}

// Whether the chain leaves a value of the input dtype unchanged: only copies
// of the running value, rounded (if at all) to the input dtype or wider.
bool identity_chain(const TransposeParams& tp) {
    if (tp.in_dtype != tp.out_dtype) return false;
    for (int k = 0; k < tp.chain.n_instr; k++) {
        const tadma_instr& I = tp.chain.prog[k];
        if (I.op != TADMA_OP_COPY || I.b == TADMA_SRC_IMM) return false;
        const int rd = I.round_dtype;
        if (rd >= 0 && rd != tp.in_dtype && rd != TADMA_F32 && rd != TADMA_F64) return false;
    }
    return true;
}

template <typename TI, typename TO, int TJ>
void launch_t16_tj(bool fast, dim3 grid, const TransposeParams& tp, cudaStream_t s) {
    if (identity_chain(tp)) (void)launch_pdl(transpose16_kernel<TI, TO, PROG_INTERP, TJ, true>, grid, dim3(THREADS), 0, s, tp);
    else if (fast) (void)launch_pdl(transpose16_kernel<TI, TO, PROG_INTERP_FAST, TJ, false>, grid, dim3(THREADS), 0, s, tp);
    else (void)launch_pdl(transpose16_kernel<TI, TO, PROG_INTERP, TJ, false>, grid, dim3(THREADS), 0, s, tp);
}
template <typename TI, typename TO>
void launch_t16_io(bool fast, int64_t gz, const TransposeParams& tp, cudaStream_t s) {
    const unsigned gy = (unsigned)((tp.n_i + 63) / 64);
    if (tp.n_j >= 256) launch_t16_tj<TI, TO, 256>(fast, dim3((unsigned)((tp.n_j + 255) / 256), gy, (unsigned)gz), tp, s);
    else launch_t16_tj<TI, TO, 128>(fast, dim3((unsigned)((tp.n_j + 127) / 128), gy, (unsigned)gz), tp, s);
}
template <typename TI>
void launch_t16_i(bool fast, int64_t gz, const TransposeParams& tp, cudaStream_t s) {
    if (tp.out_dtype == TADMA_F16) launch_t16_io<TI, __half>(fast, gz, tp, s);
    else launch_t16_io<TI, __nv_bfloat16>(fast, gz, tp, s);
}

}  // namespace

int launch_transpose(bool fast, const TransposeParams& tp, cudaStream_t s) {
    const int64_t gz = tp.nbatch < 65535 ? tp.nbatch : 65535;
    const bool in16 = tp.in_dtype == TADMA_F16 || tp.in_dtype == TADMA_BF16;
    const bool out16 = tp.out_dtype == TADMA_F16 || tp.out_dtype == TADMA_BF16;
    if (in16 && out16 && transpose64_ok(tp)) {
        if (tp.in_dtype == TADMA_F16) launch_t16_i<__half>(fast, gz > 0 ? gz : 1, tp, s);
        else launch_t16_i<__nv_bfloat16>(fast, gz > 0 ? gz : 1, tp, s);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
    }
    if (tp.in_dtype == TADMA_F32 && transpose64_ok(tp)) {
        switch (tp.out_dtype) {
        case TADMA_F32: launch_t32_o<float>(fast, gz > 0 ? gz : 1, tp, s); break;
        case TADMA_F16: launch_t32_o<__half>(fast, gz > 0 ? gz : 1, tp, s); break;
        default: launch_t32_o<__nv_bfloat16>(fast, gz > 0 ? gz : 1, tp, s); break;
        }
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
    }
    if (transpose64_ok(tp)) {
        dim3 grid((unsigned)((tp.n_j + 63) / 64), (unsigned)((tp.n_i + 63) / 64), (unsigned)(gz > 0 ? gz : 1));
        switch (tp.in_dtype) {
        case TADMA_F32: launch_t64_i<float>(fast, grid, tp, s); break;
        case TADMA_F16: launch_t64_i<__half>(fast, grid, tp, s); break;
        default: launch_t64_i<__nv_bfloat16>(fast, grid, tp, s); break;
        }
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
    }
    const int64_t gx = (tp.n_j + 31) / 32, gy = (tp.n_i + 31) / 32;
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(gz > 0 ? gz : 1));
    if (fast) (void)launch_pdl(transpose_chain_kernel<PROG_INTERP_FAST>, dim3(grid), dim3(THREADS), 0, s, tp);
    else (void)launch_pdl(transpose_chain_kernel<PROG_INTERP>, dim3(grid), dim3(THREADS), 0, s, tp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

}  // namespace tadma_b200
