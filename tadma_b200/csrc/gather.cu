// gather.cu - ONNX Gather with an optional fused broadcast add (sm_100a),
// plus the per-device error word that reports out-of-range ids.
//
// Replaces gather (Operations.hpp:244-262) + EltwiseVariadicNDNode /
// EltwiseVariadicNDKernel (kernels/EltwiseVariadicND.hpp:6-38): one scalar
// element per thread, 256-thread blocks with no bounds guard, the id re-read
// for every element, a 32-bit index (wraps above 2^32 elements) and, for
// rank-2 ids, a broken index (it writes the gathered id into idx[ids.Rank]).
// The embedding add that follows in generated graphs (gather + pos) is a
// separate CombineToNode pass over the whole output (Kernels.hpp:33-45).
//
// Fast path (axis 0, table rows contiguous): one warp per output row; the id
// is read once per row (one broadcast load, a row ahead), rows sharing an
// add row are visited together (batch-fastest), the row is copied in 8-element
// chunks (16 B of fp16/bf16, 32 B of fp32) with 4 raw chunks in flight per lane,
// the add operand's row (e.g. pos[s]) is fetched with an L2 evict_last policy
// so it stays resident across the batch; the gathered rows keep the normal
// policy, so repeated ids (a hot vocabulary subset) hit in L2, and the output
// is written with evict-first stores: the gather
// writes its output once and reads each gathered row once, so at config 5
// sizes it is an HBM-bound copy.
// Any other layout takes a per-element path with the same semantics.
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"
#include "layout.hpp"

namespace tadma_b200 {

// Per-device error word of the gather kernels (bit 1 << TADMA_ERR_INDEX = an
// id was out of range).
static __device__ unsigned int g_error_word;

namespace {

constexpr int THREADS = 256;
constexpr int CHUNK = 8;  // elements per lane step

struct GatherParams {
    const char* table;
    const char* ids;
    const char* add;
    char* out;
    int32_t t_dtype, i_dtype, a_dtype, o_dtype;
    int64_t n;  // table extent along the gather axis
    // fast path
    int64_t nrows, D, t_row_stride, o_row_stride, ids_stride;
    int32_t irank, bperm;
    DivMod idm[TADMA_MAX_RANK];  // ids dims (row -> ids multi-index)
    int64_t a_row[TADMA_MAX_RANK];  // add strides over the ids dims
    // bperm: rows are visited batch-fastest, task t -> row b * brest + q with
    // (q, b) = divmod(t, ids.dims[0]), so warps running at the same time
    // share the add operand's row (pos[s]) instead of sweeping all of it.
    DivMod bdm;
    int64_t brest;
    // generic path
    int32_t orank, ax;
    int64_t total;
    DivMod odm[TADMA_MAX_RANK];
    int64_t os[TADMA_MAX_RANK], as[TADMA_MAX_RANK], ts[TADMA_MAX_RANK], is[TADMA_MAX_RANK];
};

// Raw 8-element chunk: 1 x 16 B for 16-bit types, 2 x 16 B for fp32.  Loads
// keep the raw bits (4 or 8 registers) so UNR chunks can be in flight with a
// small register footprint; conversion happens at compute time.
template <typename T>
struct Raw8 {
    uint4 w[sizeof(T) == 4 ? 2 : 1];
};

template <typename T>
__device__ __forceinline__ void load_raw(const T* p, Raw8<T>& r, uint64_t pol) {
    r.w[0] = ld_nc_v4_policy(p, pol);
    if constexpr (sizeof(T) == 4) r.w[1] = ld_nc_v4_policy(p + 4, pol);
}

template <typename T>
__device__ __forceinline__ void raw_to_f(const Raw8<T>& r, float* f) {
    if constexpr (sizeof(T) == 4) {
        f[0] = __uint_as_float(r.w[0].x); f[1] = __uint_as_float(r.w[0].y);
        f[2] = __uint_as_float(r.w[0].z); f[3] = __uint_as_float(r.w[0].w);
        f[4] = __uint_as_float(r.w[1].x); f[5] = __uint_as_float(r.w[1].y);
        f[6] = __uint_as_float(r.w[1].z); f[7] = __uint_as_float(r.w[1].w);
    } else {
        unpack8(r.w[0], std::is_same<T, __half>::value ? TADMA_F16 : TADMA_BF16, f);
    }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float* f) {
    if constexpr (sizeof(T) == 4) {
        st_stream_v4(p, make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3])));
        st_stream_v4(p + 4, make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]), __float_as_uint(f[6]), __float_as_uint(f[7])));
    } else {
        st_stream_v4(p, pack8(f, std::is_same<T, __half>::value ? TADMA_F16 : TADMA_BF16));
    }
}

__device__ __forceinline__ int64_t load_id(const char* ids, int dt, int64_t off) {
    return dt == TADMA_I64 ? reinterpret_cast<const long long*>(ids)[off] : (int64_t)reinterpret_cast<const int32_t*>(ids)[off];
}

template <typename TT, typename AT, typename OT, bool ADD>
__global__ void __launch_bounds__(THREADS) gather_rows_kernel(const __grid_constant__ GatherParams p) {
    pdl_begin();
    constexpr int UNR = 4;
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    const int64_t nch = p.D / CHUNK;
    // The add operand (a table every batch row re-reads) is kept resident;
    // gathered rows get the normal policy: repeated ids hit in L2.  (An
    // evict_first policy here measured 4 % slower on config 5.)
    const uint64_t pol_stream = l2_policy_evict_normal();
    const uint64_t pol_keep = l2_policy_evict_last();
    auto row_of = [&](int64_t t) -> int64_t {
        if (!p.bperm) return t;
        uint64_t q, b;
        p.bdm.divmod((uint64_t)t, q, b);
        return (int64_t)b * p.brest + (int64_t)q;
    };
    // The id of the warp's next row is loaded while this row streams, so no
    // dependent id load sits in front of a row's table loads.
    int64_t row_next = row_of(gw);
    int64_t id_next = gw < p.nrows ? load_id(p.ids, p.i_dtype, row_next * p.ids_stride) : 0;
    for (int64_t t = gw; t < p.nrows; t += nw) {
        const int64_t row = row_next;
        int64_t id = id_next;
        if (t + nw < p.nrows) {
            row_next = row_of(t + nw);
            id_next = load_id(p.ids, p.i_dtype, row_next * p.ids_stride);
        }
        if (id < 0) id += p.n;
        const bool ok = (uint64_t)id < (uint64_t)p.n;
        if (!ok && lane == 0) atomicOr(&g_error_word, 1u << TADMA_ERR_INDEX);
        const TT* trow = reinterpret_cast<const TT*>(p.table) + (ok ? id : 0) * p.t_row_stride;
        const AT* arow = nullptr;
        if constexpr (ADD) {
            uint64_t e = (uint64_t)row;
            int64_t aoff = 0;
            for (int d = p.irank - 1; d >= 1; d--) {
                uint64_t q, r;
                p.idm[d].divmod(e, q, r);
                aoff += (int64_t)r * p.a_row[d];
                e = q;
            }
            aoff += (int64_t)e * p.a_row[0];
            arow = reinterpret_cast<const AT*>(p.add) + aoff;
        }
        OT* orow = reinterpret_cast<OT*>(p.out) + row * p.o_row_stride;
        for (int64_t c0 = lane; c0 < nch; c0 += 32 * UNR) {
            Raw8<TT> tr[UNR];
            Raw8<AT> ar[UNR];
#pragma unroll
            for (int u = 0; u < UNR; u++) {
                const int64_t c = c0 + 32 * u;
                if (c < nch) {
                    if (ok) load_raw<TT>(trow + c * CHUNK, tr[u], pol_stream);
                    if constexpr (ADD) load_raw<AT>(arow + c * CHUNK, ar[u], pol_keep);
                }
            }
#pragma unroll
            for (int u = 0; u < UNR; u++) {
                const int64_t c = c0 + 32 * u;
                if (c < nch) {
                    float t[CHUNK];
                    if (ok) {
                        raw_to_f<TT>(tr[u], t);
                    } else {
#pragma unroll
                        for (int j = 0; j < CHUNK; j++) t[j] = 0.0f;
                    }
                    if constexpr (ADD) {
                        float a[CHUNK];
                        raw_to_f<AT>(ar[u], a);
#pragma unroll
                        for (int j = 0; j < CHUNK; j++) t[j] = __fadd_rn(t[j], a[j]);
                    }
                    store8<OT>(orow + c * CHUNK, t);
                }
            }
        }
    }
}

__global__ void __launch_bounds__(THREADS) gather_generic_kernel(const __grid_constant__ GatherParams p) {
    pdl_begin();
    const int64_t stride = (int64_t)gridDim.x * THREADS;
    for (int64_t e0 = (int64_t)blockIdx.x * THREADS + threadIdx.x; e0 < p.total; e0 += stride) {
        int64_t idx[TADMA_MAX_RANK];
        uint64_t e = (uint64_t)e0;
        for (int d = p.orank - 1; d >= 1; d--) {
            uint64_t q, r;
            p.odm[d].divmod(e, q, r);
            idx[d] = (int64_t)r;
            e = q;
        }
        idx[0] = (int64_t)e;
        int64_t ioff = 0, ooff = 0, aoff = 0, toff = 0;
        for (int d = 0; d < p.orank; d++) {
            ooff += idx[d] * p.os[d];
            aoff += idx[d] * p.as[d];
            if (d >= p.ax && d < p.ax + p.irank) ioff += idx[d] * p.is[d - p.ax];
        }
        int64_t id = load_id(p.ids, p.i_dtype, ioff);
        if (id < 0) id += p.n;
        const bool ok = (uint64_t)id < (uint64_t)p.n;
        float v = 0.0f;
        if (ok) {
            // table index: idx[0..ax) ++ [id] ++ idx[ax+irank..)
            for (int d = 0; d < p.ax; d++) toff += idx[d] * p.ts[d];
            toff += id * p.ts[p.ax];
            for (int d = p.ax + p.irank; d < p.orank; d++) toff += idx[d] * p.ts[d - p.irank + 1];
            v = load_as<float>(p.table, p.t_dtype, toff);
        } else {
            atomicOr(&g_error_word, 1u << TADMA_ERR_INDEX);
        }
        if (p.add) v = __fadd_rn(v, load_as<float>(p.add, p.a_dtype, aoff));
        store_from(p.out, p.o_dtype, ooff, v);
    }
}

int blocks_per_sm(const void* fn) {
    static std::mutex mu;
    static std::unordered_map<const void*, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(fn);
    if (it != cache.end()) return it->second;
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, THREADS, 0) != cudaSuccess || nb <= 0) nb = 1;
    cache[fn] = nb;
    return nb;
}

template <typename TT, typename AT, typename OT, bool ADD>
int launch_rows(const GatherParams& p, cudaStream_t s) {
    // One row per warp and as many CTAs as that takes: the block scheduler
    // balances the SMs (a persistent grid-stride grid measured slower on B200).
    const int64_t want = (p.nrows + (THREADS / 32) - 1) / (THREADS / 32);
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    (void)launch_pdl(gather_rows_kernel<TT, AT, OT, ADD>, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_gather launch");
}

template <typename TT, typename AT>
int launch_out(const GatherParams& p, bool add, cudaStream_t s) {
    switch (p.o_dtype) {
    case TADMA_F32: return add ? launch_rows<TT, AT, float, true>(p, s) : launch_rows<TT, AT, float, false>(p, s);
    case TADMA_F16: return add ? launch_rows<TT, AT, __half, true>(p, s) : launch_rows<TT, AT, __half, false>(p, s);
    default: return add ? launch_rows<TT, AT, __nv_bfloat16, true>(p, s) : launch_rows<TT, AT, __nv_bfloat16, false>(p, s);
    }
}

template <typename TT>
int launch_add(const GatherParams& p, bool add, cudaStream_t s) {
    if (!add) return launch_out<TT, TT>(p, false, s);
    switch (p.a_dtype) {
    case TADMA_F32: return launch_out<TT, float>(p, true, s);
    case TADMA_F16: return launch_out<TT, __half>(p, true, s);
    default: return launch_out<TT, __nv_bfloat16>(p, true, s);
    }
}

bool is_vec_float(int dt) { return dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16; }

}  // namespace
}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" int tadma_b200_gather(const tadma_tensor* table, int32_t axis, const tadma_tensor* ids,
                                 const tadma_tensor* add, const tadma_tensor* out, void* stream) {
    std::string err = check_tensor(table, "table");
    if (err.empty()) err = check_tensor(ids, "ids");
    if (err.empty()) err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (ids->dtype != TADMA_I64 && ids->dtype != TADMA_I32) return fail(TADMA_ERR_INVALID, "ids must be int64 or int32");
    if (table->rank < 1) return fail(TADMA_ERR_INVALID, "table rank must be >= 1");
    const int ax = axis < 0 ? axis + table->rank : axis;
    if (ax < 0 || ax >= table->rank) return fail(TADMA_ERR_INVALID, "axis out of range");
    const int orank = table->rank - 1 + ids->rank;
    if (orank > TADMA_MAX_RANK) return fail(TADMA_ERR_INVALID, "output rank exceeds 8");
    if (out->rank != orank) return fail(TADMA_ERR_INVALID, "out rank must be table.rank - 1 + ids.rank");
    int64_t odims[TADMA_MAX_RANK];
    {
        int k = 0;
        for (int d = 0; d < ax; d++) odims[k++] = table->dims[d];
        for (int d = 0; d < ids->rank; d++) odims[k++] = ids->dims[d];
        for (int d = ax + 1; d < table->rank; d++) odims[k++] = table->dims[d];
        for (int d = 0; d < orank; d++)
            if (out->dims[d] != odims[d]) return fail(TADMA_ERR_INVALID, "out dims must be table[:axis] ++ ids ++ table[axis+1:]");
    }
    const bool has_add = add && add->data;
    if (has_add) {
        err = check_tensor(add, "add");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (add->rank != orank) return fail(TADMA_ERR_INVALID, "add rank must equal out rank");
        for (int d = 0; d < orank; d++)
            if (add->dims[d] != odims[d] && add->dims[d] != 1) return fail(TADMA_ERR_INVALID, "add not broadcastable to out");
    }
    if (numel(out) == 0) return TADMA_OK;
    if (table->dims[ax] == 0) return fail(TADMA_ERR_INVALID, "gather from an empty axis");

    GatherParams p{};
    p.table = (const char*)table->data;
    p.ids = (const char*)ids->data;
    p.add = has_add ? (const char*)add->data : nullptr;
    p.out = (char*)out->data;
    p.t_dtype = table->dtype;
    p.i_dtype = ids->dtype;
    p.a_dtype = has_add ? add->dtype : TADMA_F32;
    p.o_dtype = out->dtype;
    p.n = table->dims[ax];
    cudaStream_t s = (cudaStream_t)stream;
    int64_t astr[TADMA_MAX_RANK] = {};
    if (has_add)
        for (int d = 0; d < orank; d++) astr[d] = add->dims[d] == 1 ? 0 : add->strides[d];

    // Fast path: axis 0, 2-D table with contiguous rows, ids and out rows foldable.
    if (ax == 0 && table->rank == 2 && table->strides[1] == 1 && is_vec_float(table->dtype) &&
        is_vec_float(out->dtype) && (!has_add || is_vec_float(add->dtype))) {
        const int64_t D = table->dims[1];
        const int irank = ids->rank;
        // Row dims = ids dims; fold ids/out jointly over them.
        int64_t rd[TADMA_MAX_RANK], rs[2][TADMA_MAX_RANK];
        for (int d = 0; d < irank; d++) {
            rd[d] = ids->dims[d];
            rs[0][d] = ids->strides[d];
            rs[1][d] = out->strides[d];
        }
        Folded f = fold(irank, rd, rs, 2);
        const int es_t = dtype_size(table->dtype), es_o = dtype_size(out->dtype), es_a = has_add ? dtype_size(add->dtype) : 0;
        bool ok = f.rank == 1 && out->strides[orank - 1] == 1 && D % CHUNK == 0 && D > 0;
        ok = ok && (uintptr_t)table->data % 16 == 0 && (table->strides[0] * es_t) % 16 == 0;
        ok = ok && (uintptr_t)out->data % 16 == 0 && (f.strides[1][0] * es_o) % 16 == 0;
        if (has_add) {
            ok = ok && add->strides[orank - 1] == 1 && add->dims[orank - 1] == D && (uintptr_t)add->data % 16 == 0;
            for (int d = 0; d < irank && ok; d++) ok = (astr[d] * es_a) % 16 == 0;
        }
        if (ok) {
            p.nrows = f.dims[0];
            p.D = D;
            p.t_row_stride = table->strides[0];
            p.ids_stride = f.strides[0][0];
            p.o_row_stride = f.strides[1][0];
            p.irank = irank > 0 ? irank : 1;
            if (irank == 0) {
                p.idm[0] = DivMod(1);
                p.a_row[0] = 0;
            }
            for (int d = 0; d < irank; d++) {
                p.idm[d] = DivMod((uint64_t)ids->dims[d]);
                p.a_row[d] = astr[d];
            }
            // An add broadcast over the leading ids dim (pos over the batch):
            // visit rows batch-fastest so the add rows in use stay few.
            if (has_add && irank >= 2 && astr[0] == 0 && ids->dims[0] > 1) {
                p.bperm = 1;
                p.bdm = DivMod((uint64_t)ids->dims[0]);
                p.brest = p.nrows / ids->dims[0];
            }
            switch (table->dtype) {
            case TADMA_F32: return launch_add<float>(p, has_add, s);
            case TADMA_F16: return launch_add<__half>(p, has_add, s);
            default: return launch_add<__nv_bfloat16>(p, has_add, s);
            }
        }
    }
    // Generic path.
    p.orank = orank;
    p.ax = ax;
    p.irank = ids->rank;
    p.total = numel(out);
    for (int d = 0; d < orank; d++) {
        p.odm[d] = DivMod((uint64_t)out->dims[d]);
        p.os[d] = out->strides[d];
        p.as[d] = astr[d];
    }
    for (int d = 0; d < table->rank; d++) p.ts[d] = table->strides[d];
    for (int d = 0; d < ids->rank; d++) p.is[d] = ids->strides[d];
    int64_t cap = (int64_t)sm_count() * blocks_per_sm((const void*)gather_generic_kernel);
    int64_t want = (p.total + THREADS - 1) / THREADS;
    int grid = (int)(want < cap ? want : cap);
    (void)launch_pdl(gather_generic_kernel, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_gather launch");
}

extern "C" int tadma_b200_error_flags(uint32_t* flags, int32_t clear) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_error_flags sync");
    unsigned int w = 0;
    e = cudaMemcpyFromSymbol(&w, g_error_word, sizeof(w));
    if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_error_flags read");
    if (flags) *flags = w;
    if (clear) {
        unsigned int z = 0;
        e = cudaMemcpyToSymbol(g_error_word, &z, sizeof(z));
        if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_error_flags clear");
    }
    return TADMA_OK;
}
