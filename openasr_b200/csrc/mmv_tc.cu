// mmv_tc.cu -- decode GEMV (M <= 8 activation rows) on the integer tensor-core path.
//
// The decode mul_mat nodes (GgmlCpuGraphBuilder::mul_mat, cpu_graph.rs:3616-3686)
// stream every weight byte once for at most 8 activation rows.  The dp4a GEMV
// (mmv.cu) spends ~4 instructions per weight byte at M = 8; here one
// mma.sync m16n8k32 (s8 x s8 -> s32) does the 16 x 32 x 8 block dot of one
// 16-row weight tile against all 8 activation rows, so a warp issues a few
// instructions per 16 x 32 weights.  The weights go HBM -> registers -> MMA
// with no shared-memory staging (the work is HBM-bound; tcgen05 would need the
// nibbles unpacked into shared memory or TMEM first).
//
// Weights are read from a "decode tile" copy built at upload (repack kernels
// below).  A tile is 16 weight rows; a unit is one tile x one Q4_K super-block
// (256 k) or one tile x one Q8_0 block pair (64 k), laid out so that each lane
// issues contiguous 16-byte loads that land directly in its MMA A fragment:
//   Q4_K unit (2368 B): qs 4 x 512 B (load i, lane L=(g,t): row g bytes
//     [32i+8t, +8) then row g+8 bytes [32i+8t, +8) of the raw 128-byte quant
//     field) | per row 8 unpacked 6-bit scales + 8 mins (16 B x 16 rows) |
//     per row fp16 d, dmin (4 B x 16 rows)
//   Q8_0 unit (1088 B): qs 2 x 512 B (load i = block 2p+i, lane (g,t): row g
//     bytes [8t, +8) then row g+8 bytes [8t, +8)) | per row fp16 d of both
//     blocks (4 B x 16 rows)
// The MMA k order inside a block is a permutation (lane t holds quants 8t..8t+7
// of the block); the activation B fragment is loaded with the same permutation,
// so every block dot is the exact integer ggml forms.  The per-block float
// terms are then formed exactly as in mmv.cu:
//   Q8_0: acc += (float)isum * (d_w * d_a)
//   Q4_K: acc += (d_w*d_a)*(float)isum - (dmin_w*d_a)*(float)msum
// with isum = sum_j sc_j * dot_j over the 8 sub-blocks (int32) and
// msum = sum_j m_j * bsum_j, the latter from one f16 MMA of the duplicated mins
// against the 16-wide activation sums (|bsum16| <= 2032, products and sums are
// integers below 2^24, so the f32 result is exact).
#include "mma_frag.cuh"

namespace oasr {

// One CTA per 16-row tile; warp w handles super-blocks w, w + W, ... (LOOP: with the
// next unit's loads issued before the current one's MMAs; !LOOP: W >= super-blocks,
// one unit per warp, all loads issued at once).  Each super-block's terms go to shared
// memory and warp 0 adds them in super-block order (mma_frag.cuh: fold_terms).
template <int W, bool LOOP>
__global__ void __launch_bounds__(W * 32) mmv_q4k_tc_kernel(const uint8_t *__restrict__ tiles, int nsb, int64_t N,
                                                            int M, const int8_t *__restrict__ aqs,
                                                            const float *__restrict__ ad,
                                                            const int16_t *__restrict__ abs16, int K,
                                                            float *__restrict__ y, int64_t y_ld) {
    constexpr int SEGJ = TERM_SEG_BLOCKS / W;
    extern __shared__ __align__(16) float terms[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *tile = tiles + (int64_t)blockIdx.x * nsb * Q4K_UNIT;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    // weights do not depend on the previous kernel: issue them before the wait
    griddep_launch_dependents();
    Q4kUnit cur, nxt;
    if (warp < nsb) load_q4k_unit(cur, tile + (int64_t)warp * Q4K_UNIT, lane, g);
    griddep_wait();

    // B-fragment activation row g (rows past M read row 0 and are never stored)
    const int gr = g < M ? g : 0;
    const int8_t *arow = aqs + (int64_t)gr * K;
    const int16_t *brow = abs16 + (int64_t)gr * (K / 16);
    const int m0 = 2 * t, m1 = 2 * t + 1;  // C-fragment activation rows
    const int nrounds = LOOP ? (nsb + W - 1) / W : 1;
    for (int j = 0; j < nrounds; ++j) {
        const int s = j * W + warp;
        if (s < nsb) {
            if (LOOP && s + W < nsb) load_q4k_unit(nxt, tile + (int64_t)(s + W) * Q4K_UNIT, lane, g);
            const float da0 = m0 < M ? __ldg(ad + (int64_t)m0 * nsb + s) : 0.0f;
            const float da1 = m1 < M ? __ldg(ad + (int64_t)m1 * nsb + s) : 0.0f;
            q4k_unit_terms<false>(term_slot<W, 1, SEGJ>(terms, j, warp), cur, s, arow, brow, da0, da1, lane, t);
            if (LOOP && s + W < nsb) cur = nxt;
        }
        segment_end<W, 1, SEGJ>(acc, terms, j, nrounds, nsb, warp, lane);
    }
    if (warp != 0) return;
    const int64_t ra = (int64_t)blockIdx.x * TILE_ROWS + g, rb = ra + 8;
    if (m0 < M) {
        if (ra < N) y[(int64_t)m0 * y_ld + ra] = acc[0];
        if (rb < N) y[(int64_t)m0 * y_ld + rb] = acc[2];
    }
    if (m1 < M) {
        if (ra < N) y[(int64_t)m1 * y_ld + ra] = acc[1];
        if (rb < N) y[(int64_t)m1 * y_ld + rb] = acc[3];
    }
}

// Q8_0: warp w takes units w, w + W, ... (UPW of them) and issues every one of its loads
// before the wait, so a tile's weights are one round trip in flight (they do not
// depend on the predecessor).  UPW = 0 is the looping form for K past 8 units per warp:
// one unit per warp in flight ahead of the one in use.  Block terms are folded in block
// order by warp 0 as in mmv_q4k_tc_kernel.
template <int W, int UPW>
__global__ void __launch_bounds__(W * 32) mmv_q80_tc_kernel(const uint8_t *__restrict__ tiles, int npairs, int64_t N,
                                                            int M, const int8_t *__restrict__ aqs,
                                                            const float *__restrict__ ad, int K,
                                                            float *__restrict__ y, int64_t y_ld) {
    constexpr int SEGJ = TERM_SEG_BLOCKS / (2 * W);
    extern __shared__ __align__(16) float terms[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *tile = tiles + (int64_t)blockIdx.x * npairs * Q80_UNIT;
    const int nb = K / 32;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    griddep_launch_dependents();
    constexpr int NU = UPW > 0 ? UPW : 2;
    Q80Unit u[NU];
    if (UPW > 0) {
#pragma unroll
        for (int j = 0; j < NU; ++j)
            if (warp + j * W < npairs) load_q80_unit(u[j], tile + (int64_t)(warp + j * W) * Q80_UNIT, lane, g);
    } else {
        if (threadIdx.x == 0) prefetch_l2_bulk(tile, (uint32_t)npairs * Q80_UNIT);
        if (warp < npairs) load_q80_unit(u[0], tile + (int64_t)warp * Q80_UNIT, lane, g);
    }
    griddep_wait();

    const int8_t *arow = aqs + (int64_t)(g < M ? g : 0) * K;
    const int m0 = 2 * t, m1 = 2 * t + 1;
    const float *ad0 = m0 < M ? ad + (int64_t)m0 * nb : nullptr;
    const float *ad1 = m1 < M ? ad + (int64_t)m1 * nb : nullptr;
    const int nrounds = (npairs + W - 1) / W;
    if (UPW > 0) {
#pragma unroll
        for (int j = 0; j < NU; ++j) {
            if (j >= nrounds) break;  // CTA-uniform
            const int p = warp + j * W;
            if (p < npairs) q80_unit_terms<false>(term_slot<W, 2, SEGJ>(terms, j, warp), u[j], p, arow, ad0, ad1, lane, t);
            segment_end<W, 2, SEGJ>(acc, terms, j, nrounds, npairs, warp, lane);
        }
    } else {
        for (int j = 0; j < nrounds; ++j) {
            const int p = j * W + warp;
            if (p < npairs) {
                const bool more = p + W < npairs;
                if (more) load_q80_unit(u[1], tile + (int64_t)(p + W) * Q80_UNIT, lane, g);
                q80_unit_terms<false>(term_slot<W, 2, SEGJ>(terms, j, warp), u[0], p, arow, ad0, ad1, lane, t);
                if (more) u[0] = u[1];
            }
            segment_end<W, 2, SEGJ>(acc, terms, j, nrounds, npairs, warp, lane);
        }
    }
    if (warp != 0) return;
    const int64_t ra = (int64_t)blockIdx.x * TILE_ROWS + g, rb = ra + 8;
    if (m0 < M) {
        if (ra < N) y[(int64_t)m0 * y_ld + ra] = acc[0];
        if (rb < N) y[(int64_t)m0 * y_ld + rb] = acc[2];
    }
    if (m1 < M) {
        if (ra < N) y[(int64_t)m1 * y_ld + ra] = acc[1];
        if (rb < N) y[(int64_t)m1 * y_ld + rb] = acc[3];
    }
}

// ---- decode-tile repack (runs once at upload) --------------------------------------------
// get_scale_min_k4 on the 12 packed bytes (layout: gguf/quants.py Q4_K.get_scale_min)
static __device__ __forceinline__ void unpack_scale_min(const uint8_t *s, int j, int &sc, int &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// one warp per unit (tile T, super-block s); raw rows are 16-byte aligned ggml Q4_K blocks
__global__ void repack_q4k_tiles_kernel(const uint8_t *__restrict__ raw, int64_t N, int nsb, int64_t row_bytes,
                                        int64_t n_units, uint8_t *__restrict__ tiles) {
    const int lane = threadIdx.x & 31;
    const int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (unit >= n_units) return;
    const int64_t T = unit / nsb;
    const int s = (int)(unit - T * nsb);
    const int g = lane >> 2, t = lane & 3;
    uint8_t *u = tiles + unit * Q4K_UNIT;
    const int64_t ra = T * TILE_ROWS + g, rb = ra + 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint2 a = make_uint2(0, 0), b = make_uint2(0, 0);
        if (ra < N) a = *reinterpret_cast<const uint2 *>(raw + ra * row_bytes + (int64_t)s * 144 + 16 + 32 * i + 8 * t);
        if (rb < N) b = *reinterpret_cast<const uint2 *>(raw + rb * row_bytes + (int64_t)s * 144 + 16 + 32 * i + 8 * t);
        *reinterpret_cast<uint4 *>(u + i * 512 + lane * 16) = make_uint4(a.x, a.y, b.x, b.y);
    }
    if (lane < TILE_ROWS) {
        const int64_t r = T * TILE_ROWS + lane;
        uint8_t scm[16];
        uint32_t dd = 0;
        if (r < N) {
            const uint8_t *blk = raw + r * row_bytes + (int64_t)s * 144;
            for (int j = 0; j < 8; ++j) {
                int sc, m;
                unpack_scale_min(blk + 4, j, sc, m);
                scm[j] = (uint8_t)sc;
                scm[8 + j] = (uint8_t)m;
            }
            dd = *reinterpret_cast<const uint32_t *>(blk);
        } else {
            for (int j = 0; j < 16; ++j) scm[j] = 0;
        }
        uint4 v;
        memcpy(&v, scm, 16);
        *reinterpret_cast<uint4 *>(u + 2048 + 16 * lane) = v;
        *reinterpret_cast<uint32_t *>(u + 2304 + 4 * lane) = dd;
    }
}

// from the repacked Q8_0 planes: qs [N][K] int8, d [N][K/32] fp16
__global__ void repack_q80_tiles_kernel(const uint8_t *__restrict__ qs, const uint16_t *__restrict__ d, int64_t N,
                                        int K, int npairs, int64_t n_units, uint8_t *__restrict__ tiles) {
    const int lane = threadIdx.x & 31;
    const int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (unit >= n_units) return;
    const int64_t T = unit / npairs;
    const int p = (int)(unit - T * npairs);
    const int g = lane >> 2, t = lane & 3;
    uint8_t *u = tiles + unit * Q80_UNIT;
    const int64_t ra = T * TILE_ROWS + g, rb = ra + 8;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int64_t k0 = (int64_t)(2 * p + i) * 32 + 8 * t;
        uint2 a = make_uint2(0, 0), b = make_uint2(0, 0);
        if (ra < N) a = *reinterpret_cast<const uint2 *>(qs + ra * K + k0);
        if (rb < N) b = *reinterpret_cast<const uint2 *>(qs + rb * K + k0);
        *reinterpret_cast<uint4 *>(u + i * 512 + lane * 16) = make_uint4(a.x, a.y, b.x, b.y);
    }
    if (lane < TILE_ROWS) {
        const int64_t r = T * TILE_ROWS + lane;
        uint32_t v = 0;
        if (r < N) v = (uint32_t)d[r * (K / 32) + 2 * p] | ((uint32_t)d[r * (K / 32) + 2 * p + 1] << 16);
        *reinterpret_cast<uint32_t *>(u + 1024 + 4 * lane) = v;
    }
}

bool mmv_tiles_supported(int type, int64_t K) {
    if (type == OASR_TYPE_Q4_K) return K % 256 == 0;
    if (type == OASR_TYPE_Q8_0) return K % 64 == 0;
    return false;
}

size_t mmv_tiles_bytes(int type, int64_t N, int64_t K, int64_t slices) {
    const int64_t ntiles = (N + TILE_ROWS - 1) / TILE_ROWS;
    if (type == OASR_TYPE_Q4_K) return (size_t)(slices * ntiles * (K / 256) * Q4K_UNIT);
    return (size_t)(slices * ntiles * (K / 64) * Q80_UNIT);
}

cudaError_t build_mmv_tiles(oasr_weight *w, cudaStream_t st) {
    const int64_t N = w->ne[1], K = w->ne[0], slices = w->ne[2] * w->ne[3];
    const int64_t ntiles = (N + TILE_ROWS - 1) / TILE_ROWS;
    const size_t per_slice = mmv_tiles_bytes(w->type, N, K, 1);
    for (int64_t sl = 0; sl < slices; ++sl) {
        uint8_t *dst = w->tiles + sl * per_slice;
        if (w->type == OASR_TYPE_Q4_K) {
            const int nsb = (int)(K / 256);
            const int64_t units = ntiles * nsb;
            repack_q4k_tiles_kernel<<<(unsigned)((units + 7) / 8), 256, 0, st>>>(
                w->qs + sl * N * w->qs_row_bytes, N, nsb, w->qs_row_bytes, units, dst);
        } else {
            const int npairs = (int)(K / 64);
            const int64_t units = ntiles * npairs;
            repack_q80_tiles_kernel<<<(unsigned)((units + 7) / 8), 256, 0, st>>>(
                w->qs + sl * N * w->qs_row_bytes, w->d + sl * N * w->d_row_elems, N, (int)K, npairs, units, dst);
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---- launcher -------------------------------------------------------------------------
// Warps per CTA: one per unit of a tile up to 8 (Q4_K: K <= 2048 gives one super-block
// per warp); larger K loops with the next unit's loads issued ahead.
template <int W, bool LOOP>
static cudaError_t launch_q4k_w(oasr_backend *be, const uint8_t *tiles, int nsb, int64_t N, int M, const ActPlanes &a,
                                int K, float *y, int64_t y_ld) {
    const unsigned grid = (unsigned)((N + TILE_ROWS - 1) / TILE_ROWS);
    const size_t smem = term_smem_bytes<W, 1, TERM_SEG_BLOCKS / W>(nsb);
    return launch_k(be, mmv_q4k_tc_kernel<W, LOOP>, dim3(grid), dim3(W * 32), smem, tiles, nsb, N, M,
                    (const int8_t *)a.qs, (const float *)a.d, (const int16_t *)a.bs16, K, y, y_ld);
}

template <int W, int UPW>
static cudaError_t launch_q80_w(oasr_backend *be, const uint8_t *tiles, int npairs, int64_t N, int M,
                                const ActPlanes &a, int K, float *y, int64_t y_ld) {
    const unsigned grid = (unsigned)((N + TILE_ROWS - 1) / TILE_ROWS);
    const size_t smem = term_smem_bytes<W, 2, TERM_SEG_BLOCKS / (2 * W)>(npairs);
    return launch_k(be, mmv_q80_tc_kernel<W, UPW>, dim3(grid), dim3(W * 32), smem, tiles, npairs, N, M,
                    (const int8_t *)a.qs, (const float *)a.d, K, y, y_ld);
}

int launch_mmv_tc(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int M, int K, float *y,
                  int64_t y_ld) {
    const int64_t N = w->ne[1];
    const uint8_t *tiles = w->tiles + slice * mmv_tiles_bytes(w->type, N, K, 1);
    cudaError_t e;
    if (w->type == OASR_TYPE_Q4_K) {
        const int nsb = K / 256;
        // one super-block per warp up to 32 of them (K <= 8192), else 8 looping warps
        if (nsb <= 1) e = launch_q4k_w<1, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 2) e = launch_q4k_w<2, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 4) e = launch_q4k_w<4, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 5) e = launch_q4k_w<5, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 8) e = launch_q4k_w<8, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 12) e = launch_q4k_w<12, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 16) e = launch_q4k_w<16, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 20) e = launch_q4k_w<20, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 32) e = launch_q4k_w<32, false>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else e = launch_q4k_w<8, true>(be, tiles, nsb, N, M, a, K, y, y_ld);
    } else {
        const int npairs = K / 64;
        // Few tiles (N up to 4 x 16 rows per SM): every unit of a tile in flight at once --
        // 8 warps up to 8 units, 16 warps with up to 8 units each up to K = 8192.  Many
        // tiles (logits heads) or longer rows: 4 looping warps per tile behind a bulk L2
        // prefetch of the tile, the CTA count supplying the parallelism.
        const int64_t ntiles = (N + TILE_ROWS - 1) / TILE_ROWS;
        if (ntiles > 4LL * be->sm_count) e = launch_q80_w<4, 0>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else if (npairs <= 8) e = launch_q80_w<8, 1>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else if (npairs <= 16) e = launch_q80_w<16, 1>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else if (npairs <= 32) e = launch_q80_w<16, 2>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else if (npairs <= 48) e = launch_q80_w<16, 3>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else if (npairs <= 64) e = launch_q80_w<16, 4>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else if (npairs <= 128) e = launch_q80_w<16, 8>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else e = launch_q80_w<4, 0>(be, tiles, npairs, N, M, a, K, y, y_ld);
    }
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "mmv_tc launch", __LINE__);
    return oasr_internal_launch_check(be, "mmv_tc");
}

}  // namespace oasr
