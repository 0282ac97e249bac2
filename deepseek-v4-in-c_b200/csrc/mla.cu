// mla.cu - sparse MLA decode: lightning-indexer scoring, exact top-k, and
// attention over the selected latent KV rows, for a batch of sequences.
//
// Restates src/core/dsv4_indexer.c:64-106 and src/core/dsv4_attn.c:60-108.
//
// INDEXER (k_indexer_score). The selected set must equal the reference's, so
// the score is computed with the reference's own arithmetic: per head a
// SEQUENTIAL double fma chain over the head dimension, the ReLU, then heads
// folded in order as total += dot * w (product and sum rounded separately),
// and out = (float)total * scale. Same inputs, same operations, same order:
// the float scores are bit-identical, so the selection is too.
//
// TOP-K (k_topk). One CTA per sequence: radix select of the k-th key over the
// scores held in shared memory, then a bitonic sort of the chosen (value,
// index) pairs -- descending by value, ties to the lower index, exactly the
// sequence dsv4_topk's repeated argmax produces.
//
// ATTENTION (k_attn_chunk + k_attn_combine). Flash-decoding split over chunks
// of 64 selected positions: a chunk computes scores for all heads, its own
// max, exp-sums and weighted value sums; the combine rescales chunks in chunk
// order and adds the sink to the denominator only (dsv4_attn.c:84-92).
// Within one chunk this is the reference's softmax exactly; across chunks it
// agrees to float rounding.
#include <stdlib.h>

#include "common.cuh"
#include "internal.h"
#include "mla.h"

namespace dsv4b {

// Element i of a row store of type DT (compile-time, so batches of these
// loads carry no branches and issue together).
template <int DT>
__device__ __forceinline__ float load_t(const void *base, size_t i)
{
    if constexpr (DT == DSV4B_DT_F32) return __ldcg(reinterpret_cast<const float *>(base) + i);
    else if constexpr (DT == DSV4B_DT_BF16)
        return __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short *>(base) + i) << 16);
    else return e4m3x2((uint16_t)__ldcg(reinterpret_cast<const unsigned char *>(base) + i)).x;
}
template <int DT> constexpr int dt_bytes = DT == DSV4B_DT_F32 ? 4 : DT == DSV4B_DT_BF16 ? 2 : 1;

// Four consecutive elements of a row store of type DT as a float4 (the row
// offset e is a multiple of 4 and the store is aligned for it).
template <int DT>
__device__ __forceinline__ float4 load4_t(const void *base, size_t e)
{
    if constexpr (DT == DSV4B_DT_F32) return __ldcg(reinterpret_cast<const float4 *>(base) + (e >> 2));
    else if constexpr (DT == DSV4B_DT_BF16) {
        const uint2 v = __ldcg(reinterpret_cast<const uint2 *>(base) + (e >> 2));
        const float2 a = bf16x2(v.x), b = bf16x2(v.y);
        return make_float4(a.x, a.y, b.x, b.y);
    } else {
        const uint32_t v = __ldcg(reinterpret_cast<const unsigned int *>(base) + (e >> 2));
        const float2 a = e4m3x2((uint16_t)(v & 0xFFFFu)), b = e4m3x2((uint16_t)(v >> 16));
        return make_float4(a.x, a.y, b.x, b.y);
    }
}


// ---------------------------------------------------------------- indexer
constexpr int IX_TP = 32;        // positions per tile of the head-split form

// Persistent blocks (256 threads) over the batch's tiles of 32 PPL
// positions, every head; tile t of the grid-stride walk is sequence
// t / tiles, positions (t % tiles) 32 PPL .. Lane l holds positions PPL l ..
// PPL l + PPL - 1 of a tile, warp w heads 8 w .. 8 w + 7 of each group of
// 64: a register tile of PPL x 8 dots, each the sequential double FMA chain
// of the reference (src/core/dsv4_indexer.c:64-85). q sits transposed in
// shared memory ([head_dim][n_heads], loaded once per sequence; a warp reads
// its 8 heads as four 16-byte broadcasts) and the key tile as
// [head_dim][32 PPL + 2] doubles (a lane reads its PPL positions in one
// load); the next tile's keys are loaded into registers while the current
// one is computed. The per-position sum over heads in head order follows.
template <int KDT, int PPL>
__global__ void __launch_bounds__(256)
k_indexer_score(float *out, const float *q, const void *keys, long key_stride,
                long seq_key_stride, const float *w, int n_heads, int head_dim, int n_pos,
                float scale, long seq_q_stride, long seq_out_stride, const int *dyn_n, int batch, int dyn_stride)
{
    constexpr int TP = 32 * PPL, KS = TP + 2;       // tile positions, key-row stride (doubles)
    constexpr int KR = 4 * PPL;                     // key float4 groups per thread per tile (head_dim <= 128)
    pdl_trigger();
    pdl_wait();
    // rows that exist this step: one count for every sequence, or (a
    // dyn_stride) sequence b's at dyn_n[b * dyn_stride], tiles cut for the most
    const int n_launch = n_pos;
    if (dyn_n && !dyn_stride) n_pos = min(n_pos, *dyn_n);
    auto n_of = [&](int b) { return (dyn_n && dyn_stride) ? min(n_launch, dyn_n[(size_t)b * dyn_stride]) : n_pos; };
    extern __shared__ double ixs[];
    double *qt = ixs;                               // [head_dim][n_heads]
    double *kt = qt + (size_t)head_dim * n_heads;   // [head_dim][KS]
    double *dots = kt + (size_t)head_dim * KS;      // [TP][n_heads + 1]
    double *ws = dots + TP * (n_heads + 1);         // [n_heads]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nd4 = head_dim >> 2;
    const int tiles = (n_pos + TP - 1) / TP, total = tiles * batch;
    // this thread's key groups of a tile: position p = (tid >> 3) + 32 r,
    // group g = (tid & 7) + 8 u (r < PPL, u < 4)
    auto load_keys = [&](int t, float4 (&v)[KR]) {
        const int b = t / tiles, t0 = (t - b * tiles) * TP, nb = n_of(b);
        const char *kb = reinterpret_cast<const char *>(keys) + (size_t)b * seq_key_stride * dt_bytes<KDT>;
#pragma unroll
        for (int r = 0; r < PPL; r++)
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int p = (tid >> 3) + 32 * r, g = (tid & 7) + 8 * u;
                v[r * 4 + u] = (t0 + p < nb && g < nd4) ? load4_t<KDT>(kb, (size_t)(t0 + p) * key_stride + 4 * g)
                                                         : make_float4(0.f, 0.f, 0.f, 0.f);
            }
    };
    float4 kv4[KR];
    int t = blockIdx.x, qb = -1;
    if (t < total) load_keys(t, kv4);
    for (; t < total; t += gridDim.x) {
        const int b = t / tiles, t0 = (t - b * tiles) * TP;
        if (b != qb) {                              // q and w of this sequence
            qb = b;
            const float *qs = q + (size_t)b * seq_q_stride;
            for (int h = tid; h < n_heads; h += blockDim.x) ws[h] = (double)ld_act(w + (size_t)b * n_heads + h);
            const int nq4 = n_heads * nd4;
            for (int i0 = tid; i0 < nq4; i0 += 4 * (int)blockDim.x) {
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int i = i0 + u * (int)blockDim.x, h = i % n_heads, g = i / n_heads;
                    v[u] = i < nq4 ? __ldcg(reinterpret_cast<const float4 *>(qs + (size_t)h * head_dim) + g)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int i = i0 + u * (int)blockDim.x, h = i % n_heads, g = i / n_heads;
                    if (i < nq4) {
                        qt[(size_t)(4 * g) * n_heads + h] = (double)v[u].x;
                        qt[(size_t)(4 * g + 1) * n_heads + h] = (double)v[u].y;
                        qt[(size_t)(4 * g + 2) * n_heads + h] = (double)v[u].z;
                        qt[(size_t)(4 * g + 3) * n_heads + h] = (double)v[u].w;
                    }
                }
            }
        }
        // this tile's keys (loaded during the previous tile) into shared memory
#pragma unroll
        for (int r = 0; r < PPL; r++)
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int p = (tid >> 3) + 32 * r, g = (tid & 7) + 8 * u;
                if (g < nd4) {
                    const float4 v = kv4[r * 4 + u];
                    kt[(4 * g) * KS + p] = (double)v.x;
                    kt[(4 * g + 1) * KS + p] = (double)v.y;
                    kt[(4 * g + 2) * KS + p] = (double)v.z;
                    kt[(4 * g + 3) * KS + p] = (double)v.w;
                }
            }
        __syncthreads();
        if (t + (int)gridDim.x < total) load_keys(t + gridDim.x, kv4);   // in flight during the dots
        const bool vec = (n_heads & 7) == 0;        // 8 heads per warp as aligned pairs
        for (int hb = 0; hb < n_heads; hb += 64) {
            const int h0 = hb + 8 * warp;
            if (h0 >= n_heads) continue;            // warp-uniform
            double acc[PPL][8];
#pragma unroll
            for (int r = 0; r < PPL; r++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[r][j] = 0.0;
            for (int c = 0; c < head_dim; c++) {
                double kv[PPL];
                if constexpr (PPL == 2) {
                    const double2 k2 = *reinterpret_cast<const double2 *>(kt + c * KS + 2 * lane);
                    kv[0] = k2.x;
                    kv[1] = k2.y;
                } else {
                    kv[0] = kt[c * KS + lane];
                }
                const double *qr = qt + (size_t)c * n_heads + h0;
                double qv[8];
                if (vec) {
#pragma unroll
                    for (int j = 0; j < 8; j += 2) {
                        const double2 q2 = *reinterpret_cast<const double2 *>(qr + j);
                        qv[j] = q2.x;
                        qv[j + 1] = q2.y;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++) qv[j] = h0 + j < n_heads ? qr[j] : 0.0;
                }
#pragma unroll
                for (int r = 0; r < PPL; r++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[r][j] = __fma_rn(qv[j], kv[r], acc[r][j]);
            }
#pragma unroll
            for (int r = 0; r < PPL; r++)
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (h0 + j < n_heads) dots[(PPL * lane + r) * (n_heads + 1) + h0 + j] = acc[r][j];
        }
        __syncthreads();
        const int nb = n_of(b);
        for (int p = tid; p < TP; p += blockDim.x) {
            if (t0 + p >= nb) break;
            double total_s = 0.0;
            for (int h = 0; h < n_heads; h++) {
                const double d = dots[p * (n_heads + 1) + h];
                if (d > 0.0) total_s = __dadd_rn(total_s, __dmul_rn(d, ws[h]));
            }
            out[(size_t)b * seq_out_stride + t0 + p] = __fmul_rn((float)total_s, scale);
        }
        __syncthreads();                            // dots, kt and (for a new sequence) qt are reused
    }
}

// The same scores with the heads spread over blocks (decode: a few hundred
// positions would otherwise occupy a handful of SMs with long double FMA
// chains). grid (ceil(n_pos / 32), n_heads / IX_HS, batch), 256 threads:
// thread (position t & 31, head (t >> 5) of the block's IX_HS) forms the
// sequential double dot of its pair and stores term = dot > 0 ? dot * w : 0
// to terms[b][p][h]; the last block of a position tile to arrive (counter
// per tile, reset by that block) adds each position's terms in head order
// -- the reference's loop exactly, skipped heads adding +0 -- and writes out.
constexpr int IX_HS = 8;

template <int KDT>
__global__ void __launch_bounds__(256)
k_indexer_split(float *out, const float *q, const void *keys, long key_stride, long seq_key_stride, const float *w,
                int n_heads, int head_dim, int n_pos, float scale, long seq_q_stride, long seq_out_stride,
                const int *dyn_n, double *terms, unsigned *count, int dyn_stride)
{
    pdl_trigger();
    pdl_wait();
    const int n_alloc = n_pos;                      // the terms' per-sequence stride
    // rows that exist this step (sequence blockIdx.z's with a dyn_stride)
    if (dyn_n) n_pos = min(n_pos, dyn_n[(size_t)blockIdx.z * dyn_stride]);
    if ((int)blockIdx.x * IX_TP >= n_pos) return;
    extern __shared__ double ixs[];
    double *qs = ixs;                               // [IX_HS][head_dim]
    double *kt = qs + IX_HS * head_dim;             // [head_dim][IX_TP]
    __shared__ bool last;
    const int b = blockIdx.z, t0 = blockIdx.x * IX_TP, h0 = blockIdx.y * IX_HS, tid = threadIdx.x;
    const int ntiles = gridDim.x;
    q += (size_t)b * seq_q_stride + (size_t)h0 * head_dim;
    w += (size_t)b * n_heads;
    const char *kb = reinterpret_cast<const char *>(keys) + (size_t)b * seq_key_stride * dt_bytes<KDT>;
    const int nq4 = (IX_HS * head_dim) >> 2;
    for (int i = tid; i < nq4; i += blockDim.x) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(q) + i);
        qs[4 * i] = (double)v.x;
        qs[4 * i + 1] = (double)v.y;
        qs[4 * i + 2] = (double)v.z;
        qs[4 * i + 3] = (double)v.w;
    }
    {
        const int p = tid >> 3, part8 = tid & 7, nd4 = head_dim >> 2;
        const bool live = t0 + p < n_pos;
        for (int g0 = part8; g0 < nd4; g0 += 32) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int g = g0 + 8 * u;
                v[u] = (live && g < nd4) ? load4_t<KDT>(kb, (size_t)(t0 + p) * key_stride + 4 * g)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int g = g0 + 8 * u;
                if (g < nd4) {
                    kt[(4 * g) * IX_TP + p] = (double)v[u].x;
                    kt[(4 * g + 1) * IX_TP + p] = (double)v[u].y;
                    kt[(4 * g + 2) * IX_TP + p] = (double)v[u].z;
                    kt[(4 * g + 3) * IX_TP + p] = (double)v[u].w;
                }
            }
        }
    }
    __syncthreads();
    const int p = tid & 31, j = tid >> 5;
    double *tb = terms + (size_t)b * n_alloc * n_heads;
    if (t0 + p < n_pos) {
        double acc = 0.0;
        for (int c = 0; c < head_dim; c++) acc = __fma_rn(qs[j * head_dim + c], kt[c * IX_TP + p], acc);
        const double wh = (double)ld_act(w + h0 + j);
        tb[(size_t)(t0 + p) * n_heads + h0 + j] = acc > 0.0 ? __dmul_rn(acc, wh) : 0.0;
    }
    __threadfence();
    __syncthreads();
    unsigned *cnt = count + (size_t)b * ntiles + blockIdx.x;
    if (tid == 0) last = atomicAdd(cnt, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) *cnt = 0u;
    // the tile's terms into shared memory by every thread (one round of L2
    // loads, over the q tile, no longer needed), then each position's sum
    // in head order
    const int np = min(IX_TP, n_pos - t0), nt = np * n_heads;
    double *ts = ixs;                               // [np][n_heads]
    const double *tt = tb + (size_t)t0 * n_heads;
    for (int i = tid; i < nt; i += blockDim.x) ts[i] = __ldcg(tt + i);
    __syncthreads();
    if (tid < np) {
        double total = 0.0;
        for (int h = 0; h < n_heads; h++) total = __dadd_rn(total, ts[tid * n_heads + h]);
        out[(size_t)b * seq_out_stride + t0 + tid] = __fmul_rn((float)total, scale);
    }
}

// ------------------------------------------------------------------- top-k
// Orderable key: larger value -> larger key (IEEE total order on non-NaN).
__device__ __forceinline__ uint32_t fkey(float v)
{
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One CTA (1024 threads) per sequence. scores [n] -> idx [min(k, n)] in
// descending order, ties to the lower index. n <= kTopkMaxN, k <= kTopkMaxK.
__global__ void __launch_bounds__(1024)
k_topk(int *idx_out, const float *scores, int n, int k, long seq_in_stride, long seq_out_stride,
       const int *dyn_nk, int dyn_stride)
{
    pdl_trigger();
    pdl_wait();
    if (dyn_nk) {                                   // sequence blockIdx.y's {n, k} with a dyn_stride
        const int *dk = dyn_nk + (size_t)blockIdx.y * dyn_stride;
        n = min(n, dk[0]);
        k = dk[1];
    }
    extern __shared__ uint32_t tks[];
    uint32_t *key = tks;                                   // [n]
    int *eqi = reinterpret_cast<int *>(key + ((n + 1) & ~1));   // [kTopkEqCap] indices == the k-th key
    unsigned long long *sel = reinterpret_cast<unsigned long long *>(eqi + kTopkEqCap);   // [kpow2]
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_want, s_gt, s_eqtaken;
    const int b = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
    scores += (size_t)b * seq_in_stride;
    idx_out += (size_t)b * seq_out_stride;
    if (k > n) k = n;
    if (k <= 0) return;
    for (int i = tid; i < n; i += nt) key[i] = fkey(scores[i]);
    if (tid == 0) { s_prefix = 0; s_want = (uint32_t)k; }
    __syncthreads();
    // radix select, 8 bits at a time from the top: find the k-th largest key.
    // With k == n every key is taken: threshold 0 (below every non-NaN key).
    uint32_t mask = 0;
    for (int shift = 24; shift >= 0 && k < n; shift -= 8) {
        for (int i = tid; i < 256; i += nt) hist[i] = 0;
        __syncthreads();
        const uint32_t pre = s_prefix;
        // lanes with the same bin add once (float exponents cluster, and
        // unaggregated atomics on a few bins serialise)
        for (int i = tid; i < n; i += nt)
            if ((key[i] & mask) == pre) {
                const uint32_t bin = (key[i] >> shift) & 255u;
                const unsigned same = __match_any_sync(__activemask(), bin);
                if ((tid & 31) == __ffs(same) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(same));
            }
        __syncthreads();
        // the bin holding the want-th largest: lane l owns bins 255-8l .. 248-8l,
        // an exclusive scan over lanes finds the lane, the lane walks its bins
        if (tid < 32) {
            const uint32_t want = s_want;
            uint32_t cnt[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) { cnt[j] = hist[255 - 8 * tid - j]; sum += cnt[j]; }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += u;
            }
            const uint32_t excl = incl - sum;
            if (excl < want && want <= incl) {
                uint32_t acc = excl;
                int bin = 255 - 8 * tid;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (j == 7 || acc + cnt[j] >= want) { bin = 255 - 8 * tid - j; break; }
                    acc += cnt[j];
                }
                s_want = want - acc;
                s_prefix = pre | ((uint32_t)bin << shift);
            }
        }
        mask |= 255u << shift;
        __syncthreads();
    }
    if (k == n && tid == 0) s_want = 0;
    __syncthreads();
    const uint32_t kth = s_prefix;            // key of the k-th largest
    const uint32_t need_eq = s_want;          // how many == kth are taken (lowest indices)
    // count > kth, collect them; then the first need_eq indices with == kth
    if (tid == 0) { s_gt = 0; s_eqtaken = 0; }
    __syncthreads();
    int kp = 1;
    while (kp < k) kp <<= 1;
    for (int i = tid; i < kp; i += nt) sel[i] = 0ull;   // padding sorts last
    __syncthreads();
    __shared__ uint32_t s_eq;
    if (tid == 0) s_eq = 0;
    __syncthreads();
    for (int i = tid; i < n; i += nt) {
        if (key[i] > kth) {
            const uint32_t slot = atomicAdd(&s_gt, 1u);
            sel[slot] = ((unsigned long long)key[i] << 32) | (uint32_t)(~(uint32_t)i);
        } else if (key[i] == kth) {                   // ties at the threshold, in any order
            const uint32_t slot = atomicAdd(&s_eq, 1u);
            if (slot < (uint32_t)kTopkEqCap) eqi[slot] = i;
        }
    }
    __syncthreads();
    const uint32_t base = s_gt, neq = s_eq;
    if (neq <= (uint32_t)kTopkEqCap) {
        // the lowest need_eq indices of the ties: all of them when every tie
        // is taken (the final sort orders them), else those of rank < need_eq
        // (rank = how many ties have a lower index)
        for (uint32_t e = tid; e < neq; e += nt) {
            const int i = eqi[e];
            uint32_t rank = 0;
            if (neq > need_eq)
                for (uint32_t f = 0; f < neq; f++) rank += eqi[f] < i;
            if (rank < need_eq) sel[base + rank] = ((unsigned long long)kth << 32) | (uint32_t)(~(uint32_t)i);
        }
        if (tid == 0) s_eqtaken = need_eq;
        __syncthreads();
    }
    // many ties: lowest indices first -- a block-wide ordered scan
    for (int c0 = 0; c0 < n && s_eqtaken < need_eq; c0 += nt) {
        const int i = c0 + tid;
        const int is_eq = (i < n && key[i] == kth) ? 1 : 0;
        // exclusive prefix of is_eq within this pass
        __shared__ int wsum[32];
        int v = is_eq;
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, v, o);
            if ((tid & 31) >= o) v += u;
        }
        if ((tid & 31) == 31) wsum[tid >> 5] = v;
        __syncthreads();
        if (tid < 32) {
            int s = (tid < (nt >> 5)) ? wsum[tid] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, s, o);
                if (tid >= o) s += u;
            }
            wsum[tid] = s;
        }
        __syncthreads();
        const int incl = v + ((tid >> 5) ? wsum[(tid >> 5) - 1] : 0);
        const uint32_t rank = s_eqtaken + (uint32_t)(incl - is_eq);
        if (is_eq && rank < need_eq)
            sel[base + rank] = ((unsigned long long)kth << 32) | (uint32_t)(~(uint32_t)i);
        __syncthreads();
        if (tid == nt - 1) s_eqtaken += (uint32_t)incl;
        __syncthreads();
    }
    // bitonic sort, descending by (key, ~index): larger value first, and for
    // equal values the larger ~index, i.e. the lower index, first. Thread
    // pair q holds elements 2q, 2q + 1 in registers for every stage of
    // stride <= 32 (partners within the thread or the warp: shuffles); the
    // wider strides go through shared memory.
    const int npair = kp < 64 ? 32 : kp >> 1;           // warp-aligned element pairs
    auto reg_stages = [&](unsigned long long &v0, unsigned long long &v1, int q, int size, int smax) {
        for (int stride = smax; stride >= 1; stride >>= 1) {
            const bool desc = ((2 * q) & size) == 0;
            if (stride == 1) {
                const unsigned long long hi = v0 > v1 ? v0 : v1, lo = v0 > v1 ? v1 : v0;
                v0 = desc ? hi : lo;
                v1 = desc ? lo : hi;
            } else {
                const unsigned long long p0 = __shfl_xor_sync(0xffffffffu, v0, stride >> 1);
                const unsigned long long p1 = __shfl_xor_sync(0xffffffffu, v1, stride >> 1);
                const bool keep_hi = ((2 * q) < ((2 * q) ^ stride)) == desc;
                v0 = keep_hi ? (v0 > p0 ? v0 : p0) : (v0 < p0 ? v0 : p0);
                v1 = keep_hi ? (v1 > p1 ? v1 : p1) : (v1 < p1 ? v1 : p1);
            }
        }
    };
    auto reg_phase = [&](int size_lo, int size_hi, int smax) {
        for (int q0 = 0; q0 < npair; q0 += nt) {
            const int q = q0 + tid;
            if (q0 + (tid & ~31) >= npair) continue;    // whole warps only
            unsigned long long v0 = 2 * q < kp ? sel[2 * q] : 0ull, v1 = 2 * q + 1 < kp ? sel[2 * q + 1] : 0ull;
            for (int size = size_lo; size <= size_hi; size <<= 1)
                reg_stages(v0, v1, q, size, smax < (size >> 1) ? smax : (size >> 1));
            if (2 * q < kp) sel[2 * q] = v0;
            if (2 * q + 1 < kp) sel[2 * q + 1] = v1;
        }
        __syncthreads();
    };
    reg_phase(2, 64, 32);                               // every size up to 64
    for (int size = 128; size <= kp; size <<= 1) {
        for (int stride = size >> 1; stride >= 64; stride >>= 1) {
            for (int i = tid; i < kp; i += nt) {
                const int j = i ^ stride;
                if (j > i) {
                    const unsigned long long a = sel[i], c = sel[j];
                    const bool desc = ((i & size) == 0);
                    if (desc ? (a < c) : (a > c)) { sel[i] = c; sel[j] = a; }
                }
            }
            __syncthreads();
        }
        reg_phase(size, size, 32);                      // strides 32 .. 1 of this size
    }
    for (int i = tid; i < k; i += nt) idx_out[i] = (int)(~(uint32_t)(sel[i] & 0xffffffffull));
}

// --------------------------------------------------------------- attention
constexpr int AT_CH = 32;      // selected positions per chunk
constexpr int AT_HB = 16;      // heads per block
constexpr int AT_NW = 8;       // warps per block (column slices of the scores)

// Per (sequence, chunk, head) partials: chunk max pm, exp-sum pden (double)
// and the unnormalised value sum po[d]. A chunk with no valid position has
// pm = -inf and no po.
struct AttnPart {
    float *po;
    float *pm;
    double *pden;
};

// Shared memory: KV rows and q rows padded to d + 4 floats (16-byte aligned;
// for d a multiple of 32 every row starts 4 banks after the previous one, so
// the reads below are conflict-free), the per-slice partial scores [8][32][17]
// and the weights [32][16].
size_t attn_smem_bytes(int d)
{
    return ((size_t)AT_CH * (d + 4) + (size_t)AT_HB * (d + 4) + (size_t)AT_NW * AT_CH * 17 + AT_CH * AT_HB) * 4;
}

// grid (nchunk, ceil(n_heads / AT_HB), batch), 256 threads. The index list
// holds its valid entries first, so the chunks past them only mark
// themselves empty. d is a multiple of 4.
//   scores: warp w takes the float4 column groups g = w, w + 8, ...; lane
//           (pg = lane / 4, hg = lane % 4) accumulates positions pg + 8i and
//           heads hg + 4j (i, j < 4) by fma over its groups in order; the 8
//           slice sums of a (position, head) are then added in slice order;
//   softmax: per head over the chunk's valid positions: max, expf, exp-sum in
//           double (the sink is added by k_attn_combine);
//   values:  a thread owns columns c and c + 256 for all 16 heads, fma over
//           the positions in order (masked rows are zero in shared memory).
template <int KDT>
__global__ void __launch_bounds__(256)
k_attn_chunk(AttnPart part, const float *q, const void *kv, long seq_kv_rows,
             const int *idxs, long seq_idx_stride, int n_heads, int d, int topk, float scale,
             long seq_q_stride)
{
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float ats[];
    const int dp = d + 4, nd4 = d >> 2;
    float *kvs = ats;                                       // [AT_CH][dp]
    float *qs = kvs + AT_CH * dp;                           // [AT_HB][dp]
    float *ps = qs + AT_HB * dp;                            // [AT_NW][AT_CH][17]
    float *scT = ps + AT_NW * AT_CH * 17;                   // [AT_CH][AT_HB]: weights
    __shared__ int pidx[AT_CH];
    const int b = blockIdx.z, nch = gridDim.x, c0 = blockIdx.x * AT_CH, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int h0 = blockIdx.y * AT_HB, nh = min(AT_HB, n_heads - h0);
    q += (size_t)b * seq_q_stride + (size_t)h0 * d;
    idxs += (size_t)b * seq_idx_stride;
    const char *kvb = reinterpret_cast<const char *>(kv) + (size_t)b * seq_kv_rows * d * dt_bytes<KDT>;
    const int npos = min(AT_CH, topk - c0);
    const int pi = (tid < npos) ? __ldcg(idxs + c0 + tid) : -1;
    if (tid < AT_CH) pidx[tid] = pi;
    const size_t prow = ((size_t)b * nch + blockIdx.x) * n_heads + h0;
    if (!__syncthreads_or(tid < AT_CH && pi >= 0)) {
        if (tid < nh) {
            part.pm[prow + tid] = -INFINITY;
            part.pden[prow + tid] = 0.0;
        }
        return;
    }
    // KV rows: thread (row tid / 8, lane group tid % 8) moves float4 groups
    // tid % 8 + 8k of its row, up to 16 loads in flight; masked rows are
    // zero-filled
    {
        const int p = tid >> 3, part8 = tid & 7, r = pidx[p];
        for (int g0 = part8; g0 < nd4; g0 += 128) {
            float4 v[16];
#pragma unroll
            for (int u = 0; u < 16; u++) {
                const int g = g0 + 8 * u;
                v[u] = (r >= 0 && g < nd4) ? load4_t<KDT>(kvb, (size_t)r * d + 4 * g) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 16; u++) {
                const int g = g0 + 8 * u;
                if (g < nd4) *reinterpret_cast<float4 *>(kvs + p * dp + 4 * g) = v[u];
            }
        }
    }
    // the block's q rows (zero past n_heads)
    {
        const int n4 = AT_HB * nd4;
        for (int i0 = tid; i0 < n4; i0 += 8 * (int)blockDim.x) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = i0 + u * (int)blockDim.x, h = i / nd4;
                v[u] = (i < n4 && h < nh) ? __ldcg(reinterpret_cast<const float4 *>(q) + i)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = i0 + u * (int)blockDim.x;
                if (i < n4) {
                    const int h = i / nd4, g = i - h * nd4;
                    *reinterpret_cast<float4 *>(qs + h * dp + 4 * g) = v[u];
                }
            }
        }
    }
    __syncthreads();
    // scores, slice sums
    {
        const int pg = lane >> 2, hg = lane & 3;
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
        for (int g = warp; g < nd4; g += AT_NW) {
            float4 kq[4], qq[4];
#pragma unroll
            for (int i = 0; i < 4; i++) kq[i] = *reinterpret_cast<const float4 *>(kvs + (pg + 8 * i) * dp + 4 * g);
#pragma unroll
            for (int j = 0; j < 4; j++) qq[j] = *reinterpret_cast<const float4 *>(qs + (hg + 4 * j) * dp + 4 * g);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float t = acc[i][j];
                    t = __fmaf_rn(qq[j].x, kq[i].x, t);
                    t = __fmaf_rn(qq[j].y, kq[i].y, t);
                    t = __fmaf_rn(qq[j].z, kq[i].z, t);
                    t = __fmaf_rn(qq[j].w, kq[i].w, t);
                    acc[i][j] = t;
                }
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) ps[(warp * AT_CH + pg + 8 * i) * 17 + hg + 4 * j] = acc[i][j];
    }
    __syncthreads();
    // softmax: warp w takes heads 2w, 2w + 1; lane = position
    {
        const int p = lane;
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const int h = 2 * warp + hh;
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < AT_NW; w++) acc = __fadd_rn(acc, ps[(w * AT_CH + p) * 17 + h]);
            const float s = (pidx[p] >= 0) ? __fmul_rn(acc, scale) : -INFINITY;
            const float m = warp_max_f(s);
            const float e = (m == -INFINITY || s == -INFINITY) ? 0.0f : expf(s - m);
            const double ds = warp_sum_d((double)e);
            scT[p * AT_HB + h] = e;
            if (p == 0 && h < nh) {
                part.pm[prow + h] = m;
                part.pden[prow + h] = ds;
            }
        }
    }
    __syncthreads();
    // unnormalised value sums
    for (int cb = tid; cb < d; cb += 2 * (int)blockDim.x) {
        const int c1 = cb + (int)blockDim.x;
        const bool two = c1 < d;
        float o0[AT_HB], o1[AT_HB];
#pragma unroll
        for (int h = 0; h < AT_HB; h++) o0[h] = o1[h] = 0.0f;
#pragma unroll 2
        for (int pp = 0; pp < AT_CH; pp++) {
            const float4 *e4 = reinterpret_cast<const float4 *>(scT + pp * AT_HB);
            const float4 ea = e4[0], eb = e4[1], ec = e4[2], ed = e4[3];
            const float e[AT_HB] = {ea.x, ea.y, ea.z, ea.w, eb.x, eb.y, eb.z, eb.w,
                                    ec.x, ec.y, ec.z, ec.w, ed.x, ed.y, ed.z, ed.w};
            const float v0 = kvs[pp * dp + cb], v1 = two ? kvs[pp * dp + c1] : 0.0f;
#pragma unroll
            for (int h = 0; h < AT_HB; h++) {
                o0[h] = __fmaf_rn(e[h], v0, o0[h]);
                o1[h] = __fmaf_rn(e[h], v1, o1[h]);
            }
        }
#pragma unroll
        for (int h = 0; h < AT_HB; h++)
            if (h < nh) {
                part.po[(prow + h) * d + cb] = o0[h];
                if (two) part.po[(prow + h) * d + c1] = o1[h];
            }
    }
}

// grid (n_heads, ceil(d / 128), batch), 128 threads, one output column per
// thread: rescale chunks in chunk order, add the sink to the denominator
// only, normalise. Every block works out the chunk factors of its head (a
// few hundred values at most) and the list of live chunks (pm > -inf) in
// order; empty chunks are skipped.
constexpr int AT_MAXCH = 512;

__global__ void __launch_bounds__(128)
k_attn_combine(float *o, AttnPart part, const float *sink, int nch, int n_heads, int d, long seq_o_stride,
               AttnRope rope)
{
    pdl_trigger();
    pdl_wait();
    __shared__ float fac[AT_MAXCH];
    __shared__ short lst[AT_MAXCH];
    __shared__ double dterm[AT_MAXCH];
    __shared__ float s_inv, s_M;
    __shared__ int s_nl;
    const int h = blockIdx.x, b = blockIdx.z, tid = threadIdx.x, cb0 = blockIdx.y * 128;
    float *ob = o + (size_t)b * seq_o_stride + (size_t)h * d;
    const size_t r0 = (size_t)b * nch * n_heads + h;
    if (tid < 32) {
        float M = -INFINITY;
        for (int c = tid; c < nch; c += 32) {
            const float mc = ld_act(part.pm + r0 + (size_t)c * n_heads);
            fac[c] = mc;
            M = fmaxf(M, mc);
        }
        M = warp_max_f(M);
        __syncwarp();
        int base = 0;
        for (int c0 = 0; c0 < nch; c0 += 32) {
            const int c = c0 + tid;
            const float mc = c < nch ? fac[c] : -INFINITY;
            const bool lv = mc != -INFINITY;
            if (c < nch) {
                dterm[c] = lv ? ld_act_d(part.pden + r0 + (size_t)c * n_heads) * (double)expf(mc - M) : 0.0;
                fac[c] = lv ? ((mc == M) ? 1.0f : expf(mc - M)) : 0.0f;
            }
            const unsigned live = __ballot_sync(0xffffffffu, lv);
            if (lv) lst[base + __popc(live & ((1u << tid) - 1u))] = (short)c;
            base += __popc(live);
        }
        __syncwarp();
        if (tid == 0) {
            s_M = M;
            s_nl = base;
            if (M != -INFINITY) {
                double den = 0.0;
                for (int k = 0; k < base; k++) den += dterm[lst[k]];
                den += (double)expf(sink[h] - M);
                s_inv = (float)(1.0 / den);
            }
        }
    }
    __syncthreads();
    const int cc = cb0 + tid;
    if (s_M == -INFINITY) {       // nothing valid: zero output (dsv4_attn.c:32-37)
        if (cc < d) ob[cc] = 0.0f;
        return;
    }
    const int nl = s_nl;
    if (cc < d) {
        const float *pc = part.po + r0 * d + cc;
        const size_t cstride = (size_t)n_heads * d;
        float acc = 0.0f;
        for (int k0 = 0; k0 < nl; k0 += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = k0 + u < nl ? ld_act(pc + (size_t)lst[k0 + u] * cstride) : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (k0 + u < nl) acc = __fadd_rn(acc, __fmul_rn(v[u], fac[lst[k0 + u]]));
        }
        ob[cc] = __fmul_rn(acc, s_inv);
    }
    if (rope.cs) {          // de-rotate this block's part of the tail (src/model/dsv4_layer.c:303-305)
        __syncthreads();
        const int half = rope.rd / 2, pos = __ldcg(rope.pos + (size_t)b * rope.pos_stride), t0 = d - rope.rd;
        for (int i = tid; i < half; i += blockDim.x) {
            const int e0 = t0 + 2 * i;
            if (e0 < cb0 || e0 >= cb0 + 128) continue;
            const float re = ob[e0], im = ob[e0 + 1];
            const float ci = rope.cs[(size_t)pos * half + i], si = -rope.sn[(size_t)pos * half + i];
            ob[e0] = __fsub_rn(__fmul_rn(re, ci), __fmul_rn(im, si));
            ob[e0 + 1] = __fadd_rn(__fmul_rn(re, si), __fmul_rn(im, ci));
        }
    }
}

// ------------------------------------------------------------------ launch

int indexer_score(float *out, const float *q, const void *keys, int key_dt, long key_stride,
                  long seq_key_stride, const float *w, int n_heads, int head_dim, int n_pos, float scale,
                  int batch, cudaStream_t st, const int *dyn_n, double *terms, unsigned *count, int dyn_stride)
{
    if (n_pos <= 0 || batch <= 0) return 0;
    if (terms && count && n_heads % IX_HS == 0 && head_dim % 4 == 0 && (key_stride & 3) == 0 &&
        (seq_key_stride & 3) == 0 && ((uintptr_t)q & 15) == 0 &&
        (uintptr_t)keys % (key_dt == DSV4B_DT_F32 ? 16 : key_dt == DSV4B_DT_BF16 ? 8 : 4) == 0) {
        size_t sm = ((size_t)IX_HS * head_dim + (size_t)head_dim * IX_TP) * 8;
        if ((size_t)IX_TP * n_heads * 8 > sm) sm = (size_t)IX_TP * n_heads * 8;
        if (sm <= 200 * 1024) {
            if (smem_optin(k_indexer_split<DSV4B_DT_F32>, 200 * 1024) ||
                smem_optin(k_indexer_split<DSV4B_DT_BF16>, 200 * 1024) ||
                smem_optin(k_indexer_split<DSV4B_DT_E4M3>, 200 * 1024))
                return -1;
            const dim3 grid((n_pos + IX_TP - 1) / IX_TP, n_heads / IX_HS, batch);
            const long sq = (long)n_heads * head_dim;
            if (key_dt == DSV4B_DT_F32)
                launch(k_indexer_split<DSV4B_DT_F32>, grid, dim3(256), sm, st, out, q, keys, key_stride,
                       seq_key_stride, w, n_heads, head_dim, n_pos, scale, sq, (long)n_pos, dyn_n, terms, count,
                       dyn_stride);
            else if (key_dt == DSV4B_DT_BF16)
                launch(k_indexer_split<DSV4B_DT_BF16>, grid, dim3(256), sm, st, out, q, keys, key_stride,
                       seq_key_stride, w, n_heads, head_dim, n_pos, scale, sq, (long)n_pos, dyn_n, terms, count,
                       dyn_stride);
            else
                launch(k_indexer_split<DSV4B_DT_E4M3>, grid, dim3(256), sm, st, out, q, keys, key_stride,
                       seq_key_stride, w, n_heads, head_dim, n_pos, scale, sq, (long)n_pos, dyn_n, terms, count,
                       dyn_stride);
            return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
        }
    }
    // float4 groups of q and of key rows
    const int kal = key_dt == DSV4B_DT_F32 ? 16 : key_dt == DSV4B_DT_BF16 ? 8 : 4;
    if ((head_dim & 3) || (key_stride & 3) || (seq_key_stride & 3) || ((uintptr_t)keys % kal) ||
        ((uintptr_t)q & 15))
        return -1;
    // 64 positions per tile where q, the key tile and the dots fit, else 32;
    // one persistent block per SM (two where they fit) over every tile
    if (head_dim > 128) return -1;
    auto smem_of = [&](int ppl) {
        const size_t tp = 32 * (size_t)ppl;
        return ((size_t)n_heads * head_dim + (size_t)head_dim * (tp + 2) + tp * (n_heads + 1) + (size_t)n_heads) * 8;
    };
    const int ppl = smem_of(2) <= 200 * 1024 ? 2 : 1;
    const size_t smem = smem_of(ppl);
    if (smem > 200 * 1024) return -1;
    const long sq = (long)n_heads * head_dim;
    int dev = 0, nsm = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const long tiles = ((long)n_pos + 32 * ppl - 1) / (32 * ppl) * batch;
    const long cap = (long)nsm * (smem <= 110 * 1024 ? 2 : 1);
    const dim3 grid((unsigned)(tiles < cap ? tiles : cap));
#define DSV4B_IX_LAUNCH(KDT, PPL)                                                                                 \
    do {                                                                                                         \
        if (smem_optin(k_indexer_score<KDT, PPL>, 200 * 1024)) return -1;                                        \
        launch(k_indexer_score<KDT, PPL>, grid, dim3(256), smem, st, out, q, keys, key_stride, seq_key_stride, w, \
               n_heads, head_dim, n_pos, scale, sq, n_pos, dyn_n, batch, dyn_stride);                            \
    } while (0)
    if (key_dt == DSV4B_DT_F32) {
        if (ppl == 2) DSV4B_IX_LAUNCH(DSV4B_DT_F32, 2); else DSV4B_IX_LAUNCH(DSV4B_DT_F32, 1);
    } else if (key_dt == DSV4B_DT_BF16) {
        if (ppl == 2) DSV4B_IX_LAUNCH(DSV4B_DT_BF16, 2); else DSV4B_IX_LAUNCH(DSV4B_DT_BF16, 1);
    } else {
        if (ppl == 2) DSV4B_IX_LAUNCH(DSV4B_DT_E4M3, 2); else DSV4B_IX_LAUNCH(DSV4B_DT_E4M3, 1);
    }
#undef DSV4B_IX_LAUNCH
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int topk(int *idx, const float *scores, int n, int k, int batch, long seq_in_stride, long seq_out_stride,
         cudaStream_t st, const int *dyn_nk, int dyn_stride)
{
    if (batch <= 0 || n <= 0 || k <= 0) return 0;
    if (n > kTopkMaxN || k > kTopkMaxK) return -1;
    int kp = 1;
    while (kp < (k < n ? k : n)) kp <<= 1;
    const size_t smem = (size_t)((n + 1) & ~1) * 4 + (size_t)kTopkEqCap * 4 + (size_t)kp * 8;
    if (smem > 220 * 1024) return -1;
    if (smem_optin(k_topk, 220 * 1024)) return -1;
    launch(k_topk, dim3(dim3(1, batch)), dim3(1024), smem, st, idx, scores, n, k, seq_in_stride, seq_out_stride, dyn_nk,
           dyn_stride);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

size_t attn_part_bytes(int n_heads, int d, int topk, int batch)
{
    const size_t nch = (topk + AT_CH - 1) / AT_CH;
    return (size_t)batch * nch * n_heads * ((size_t)d * 4 + 4 + 8) + 64;
}

int sparse_attn(float *o, const float *q, const void *kv, int kv_dt, long seq_kv_rows, const float *sink,
                const int *idxs, long seq_idx_stride, int n_heads, int d, int topk, float scale, int batch,
                void *part_buf, cudaStream_t st, const AttnRope *rope)
{
    if (batch <= 0 || topk <= 0) return 0;
    if (n_heads <= 0 || d > 1024 || (d & 3)) return -1;
    const int nch = (topk + AT_CH - 1) / AT_CH;
    if (nch > AT_MAXCH) return -1;
    const size_t n = (size_t)batch * nch * n_heads;
    AttnPart part;
    part.pden = reinterpret_cast<double *>(part_buf);
    part.pm = reinterpret_cast<float *>(part.pden + n);
    part.po = part.pm + n + (n & 1);
    const size_t smem = attn_smem_bytes(d);
    if (smem > 220 * 1024) return -1;
    if (smem_optin(k_attn_chunk<DSV4B_DT_F32>, 220 * 1024) || smem_optin(k_attn_chunk<DSV4B_DT_BF16>, 220 * 1024) ||
        smem_optin(k_attn_chunk<DSV4B_DT_E4M3>, 220 * 1024))
        return -1;
    const dim3 grid(nch, (n_heads + AT_HB - 1) / AT_HB, batch);
    const long sq = (long)n_heads * d;
    if (kv_dt == DSV4B_DT_F32)
        launch(k_attn_chunk<DSV4B_DT_F32>, grid, dim3(256), smem, st, part, q, kv, seq_kv_rows, idxs, seq_idx_stride,
               n_heads, d, topk, scale, sq);
    else if (kv_dt == DSV4B_DT_BF16)
        launch(k_attn_chunk<DSV4B_DT_BF16>, grid, dim3(256), smem, st, part, q, kv, seq_kv_rows, idxs, seq_idx_stride,
               n_heads, d, topk, scale, sq);
    else
        launch(k_attn_chunk<DSV4B_DT_E4M3>, grid, dim3(256), smem, st, part, q, kv, seq_kv_rows, idxs, seq_idx_stride,
               n_heads, d, topk, scale, sq);
    const AttnRope rp = rope ? *rope : AttnRope{nullptr, nullptr, nullptr, 0};
    launch(k_attn_combine, dim3(n_heads, (d + 127) / 128, batch), dim3(128), 0, st, o, part, sink, nch, n_heads, d,
           (long)n_heads * d, rp);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace dsv4b
