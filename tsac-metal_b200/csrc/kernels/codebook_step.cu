// Fused codebook step (codebook_step.cuh): one cluster of 4 CTAs = 4 heads
// per 8 rows, 256 threads per CTA.
//
// Phases of a CTA of rank c (the cluster's head c), rows r of its cluster:
//   input    book 0: h = cond row + position;  book > 0: embeddings -> BF8L ->
//            proj61 outputs [128c, 128c+128) + position -> exchange -> h
//   layer    LN1(h) -> BF8L (every CTA, all rows)
//            QKV outputs of head c -> q (shared memory), k, v (cache)
//            attention of head c (two 128-thread groups, one row each)
//            exchange -> BF8L of the 512 attention outputs
//            out-projection [128c, +128) + residual -> exchange -> h
//            LN2(h) -> BF8L; FFN-in [512c, +512) + GELU -> BF8L of its two
//            256-blocks -> exchange -> FFN-out [128c, +128) + residual ->
//            exchange -> h
//   output   final LN -> BF8L; logits [256c, +256) -> exchange; softmax and
//            bisection masses of rows r = c, c + 4 (full logit rows from the
//            four CTAs).
// Linear layers use the int8 tensor-core split of qlinear.cu's decode kernel
// (mma.sync m16n8k32, exact int32 block dots) with each warp owning whole
// 16-feature tiles, so the ordered block fold happens in registers.  Every
// CTA of a cluster executes the same sequence of cluster barriers.
#include "kernels/codebook_step.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"
#include "kernels/row_ops.cuh"

#include <cooperative_groups.h>

#include <mutex>

namespace cg = cooperative_groups;

namespace tsacb::dev
{
namespace
{
constexpr int CL = 4;                  // CTAs per cluster (= attention heads)
constexpr int R = CODEBOOK_STEP_ROWS;  // rows per cluster (one 8-row m-tile)
constexpr int THREADS = 256;
constexpr int XQ_STRIDE = 2048 + 64;   // bytes per quantized row: rows 64 bytes apart mod 128 (no bank conflicts)

// A 128-thread attention group's shared memory for at most 16 keys (the
// codebook stack attends to at most 12).
struct SmallAttention
{
    unsigned ks[16][65];
    unsigned vs[16][65];
    float q[ATT_HW];
    float scores[16];
    AttArgMax warp_best[2];
    float block_sum;
};

// Per-warp double buffer of weight chunks: 16 rows (one feature tile) x 512
// bytes (two 256-blocks), filled by bulk copies that complete on an mbarrier.
constexpr int CHUNK = 16 * 512;
struct __align__(16) WeightRing
{
    std::int8_t slot[THREADS / 32][2][CHUNK];
    unsigned long long full[THREADS / 32][2];
};

struct __align__(16) StepShared
{
    std::int8_t xq[R][XQ_STRIDE];      // quantized input rows of the next linear
    float xs[R][8];                     // their block scales
    std::uint16_t h[R][512];            // residual rows (full, every CTA)
    std::uint16_t stage[R][1024];       // bf16 staging (embeddings, FFN-in slice, logit rows)
    // Read by the cluster's other CTAs:
    std::uint16_t att_out[R][ATT_HW];   // this head's attention output
    std::uint16_t h_slice[R][128];      // this CTA's columns of a residual update
    std::int8_t mlp_q[R][512];          // this CTA's FFN-in outputs, BF8L
    float mlp_s[R][2];
    std::uint16_t logit_slice[R][256];
    // Local:
    std::uint16_t q_head[R][ATT_HW];
    SmallAttention att[2];
    SoftmaxShared soft;
    WeightRing ring;
};

__device__ __forceinline__ void mma_s8(int (&d)[4], unsigned a0, unsigned a1, unsigned a2,
                                       unsigned a3, unsigned b0, unsigned b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32"
                 " {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ std::uint32_t smem_addr(const void* p)
{
    return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool ring_try(std::uint32_t bar, std::uint32_t parity)
{
    std::uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Bounded wait (about one second of global time); false on timeout.
__device__ __forceinline__ bool ring_wait(std::uint32_t bar, std::uint32_t parity)
{
    if (ring_try(bar, parity))
        return true;
    unsigned long long start;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
    for (unsigned i = 1;; ++i)
    {
        if (ring_try(bar, parity))
            return true;
        if ((i & 63u) == 0)
        {
            unsigned long long now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (now - start > 1000000000ull)
                return false;
        }
    }
}

// Bulk copy of the weight chunk (tile n0, bytes [k0, k0 + 512) of 16 rows)
// into a warp slot; lane 0 arms the barrier, lanes 0..15 copy one row each
// (one 8 KB copy when the 16 rows are contiguous).
__device__ __forceinline__ void issue_chunk(const std::int8_t* weights, int k, int n0, int k0,
                                            std::int8_t* slot, std::uint32_t bar, int lane)
{
    if (lane == 0)
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(CHUNK)
                     : "memory");
    __syncwarp();
    // The slot's previous contents were read through the generic proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (k == 512)
    {
        if (lane == 0)
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                             smem_addr(slot)),
                         "l"(weights + static_cast<size_t>(n0) * k), "r"(CHUNK), "r"(bar)
                         : "memory");
    }
    else if (lane < 16)
    {
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_addr(slot + lane * 512)),
                     "l"(weights + static_cast<size_t>(n0 + lane) * k + k0), "r"(512), "r"(bar)
                     : "memory");
    }
}

// One CTA's share of a linear layer over the cluster's R rows: `tiles`
// 16-feature tiles (tile i starts at feature tile_n0(i)), K = k from the
// quantized rows in shared memory.  Warp w owns tiles w, w + 8, ...; its
// weights stream through the warp's two ring slots in 512-byte K spans, the
// next span's bulk copy in flight while the current one is used.  Per tile
// the 256-blocks are taken in order and each block's exact int32 dots are
// folded at once: sum = fma(dot, w_scale * x_scale, sum).  epi(m, n, sum) is
// called for every (row, feature) of the tile.  `phase` counts the uses of
// the warp's ring barriers across calls (both slots advance together).
template <class TileN0, class Epi>
__device__ __forceinline__ void cta_linear(const CodebookLinear& L, int n_total, int k, int tiles,
                                           TileN0 tile_n0, StepShared& sh, unsigned& ring_uses,
                                           bool& timed_out, Epi epi)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int spans = k / 512; // chunks per tile
    const int my_tiles = tiles > warp ? (tiles - warp + THREADS / 32 - 1) / (THREADS / 32) : 0;
    const int chunks = my_tiles * spans;
    std::int8_t* slots[2] = {sh.ring.slot[warp][0], sh.ring.slot[warp][1]};
    const std::uint32_t bars[2] = {smem_addr(&sh.ring.full[warp][0]), smem_addr(&sh.ring.full[warp][1])};
    auto chunk_tile = [&](int c) { return tile_n0(warp + (c / spans) * (THREADS / 32)); };
    // Chunk c of this call uses slot (ring_uses + c) & 1.
    for (int c = 0; c < chunks && c < 2; ++c)
    {
        const int u = static_cast<int>(ring_uses) + c;
        issue_chunk(L.weights, k, chunk_tile(c), (c % spans) * 512, slots[u & 1], bars[u & 1], lane);
    }
    float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c = 0; c < chunks; ++c)
    {
        const int u = static_cast<int>(ring_uses) + c;
        const int s = u & 1;
        const int n0 = chunk_tile(c), span = c % spans;
        // This lane's weight scales for the chunk's two blocks, loaded while
        // the chunk's copy completes.
        float wsc[2][2];
#pragma unroll
        for (int bl = 0; bl < 2; ++bl)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
                wsc[bl][hh] = __ldg(L.scales + (span * 2 + bl) * n_total + n0 + g + 8 * hh);
        if (!ring_wait(bars[s], static_cast<std::uint32_t>(u >> 1) & 1u))
            timed_out = true;
        const std::int8_t* wa = slots[s] + g * 512 + t * 16;
        const std::int8_t* wb = wa + 8 * 512;
        const std::int8_t* xa = &sh.xq[g][span * 512 + t * 16];
#pragma unroll
        for (int bl = 0; bl < 2; ++bl)
        {
            const int b = span * 2 + bl;
            int d[4] = {0, 0, 0, 0};
#pragma unroll
            for (int q = 0; q < 4; ++q)
            {
                const uint4 alo = *reinterpret_cast<const uint4*>(wa + bl * 256 + q * 64);
                const uint4 ahi = *reinterpret_cast<const uint4*>(wb + bl * 256 + q * 64);
                const uint4 xv = *reinterpret_cast<const uint4*>(xa + bl * 256 + q * 64);
                mma_s8(d, alo.x, ahi.x, alo.y, ahi.y, xv.x, xv.y);
                mma_s8(d, alo.z, ahi.z, alo.w, ahi.w, xv.z, xv.w);
            }
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
            {
                const int m = 2 * t + (cc & 1);
                const float scale = __fmul_rn(wsc[bl][cc >> 1], sh.xs[m][b]);
                sum[cc] = __fmaf_rn(static_cast<float>(d[cc]), scale, sum[cc]);
            }
        }
        __syncwarp();
        if (c + 2 < chunks)
            issue_chunk(L.weights, k, chunk_tile(c + 2), ((c + 2) % spans) * 512, slots[s], bars[s], lane);
        if (span == spans - 1)
        {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
                epi(2 * t + (cc & 1), n0 + g + 8 * (cc >> 1), sum[cc]);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
                sum[cc] = 0.0f;
        }
    }
    ring_uses += static_cast<unsigned>(chunks);
}

__device__ __forceinline__ std::uint16_t add_bf16(std::uint16_t a, std::uint16_t b)
{
    return to_bf16(__fadd_rn(from_bf16(a), from_bf16(b)));
}

__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(THREADS, 1)
    codebook_step_kernel(const CodebookStepArgs a)
{
    extern __shared__ __align__(16) unsigned char step_smem[];
    StepShared& sh = *reinterpret_cast<StepShared*>(step_smem);
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int row0 = static_cast<int>(blockIdx.x / CL) * R;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    StepShared* peer[CL];
#pragma unroll
    for (int p = 0; p < CL; ++p)
        peer[p] = cluster.map_shared_rank(&sh, p);
    auto valid = [&](int r) { return row0 + r < a.rows; };
    bool finite = true, timed_out = false;
    unsigned ring_uses = 0; // this warp's ring barrier uses so far
    if (tid == 0)
    {
        for (int w = 0; w < THREADS / 32; ++w)
            for (int s2 = 0; s2 < 2; ++s2)
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&sh.ring.full[w][s2])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // Gather the residual rows from the four CTAs' slices.
    auto gather_h = [&]()
    {
        for (int i = tid; i < R * 64; i += THREADS) // 16-byte pieces: 64 per row
        {
            const int r = i >> 6, piece = i & 63, owner = piece >> 4;
            *reinterpret_cast<uint4*>(&sh.h[r][piece * 8]) =
                *reinterpret_cast<const uint4*>(&peer[owner]->h_slice[r][(piece & 15) * 8]);
        }
    };
    // BF8L of bf16 rows held as 256-value blocks; task (r, b) reads its block
    // through `src(r, b, lane)` (8 values per lane) into xq / xs.
    auto quantize_rows = [&](int blocks, auto src)
    {
        for (int task = warp; task < R * blocks; task += THREADS / 32)
        {
            const int r = task / blocks, b = task % blocks;
            const uint4 raw = src(r, b, lane);
            bool ok = true;
            const Bf8lLane q = bf8l_block(raw, ok);
            finite = finite && (ok || !valid(r));
            *reinterpret_cast<uint2*>(&sh.xq[r][b * 256 + lane * 8]) = make_uint2(q.packed[0], q.packed[1]);
            if (lane == 0)
                sh.xs[r][b] = q.scale;
        }
    };
    auto layer_norm_rows = [&](int norm)
    {
        if (warp < R)
        {
            const bool ok = layer_norm_row(sh.h[warp], a.norm_gain[norm], a.norm_bias[norm], nullptr,
                                           sh.xq[warp], sh.xs[warp]);
            finite = finite && (ok || !valid(warp));
        }
    };

    // ------------------------------------------------------------- input --
    if (a.book == 0)
    {
        for (int i = tid; i < R * 256; i += THREADS)
        {
            const int r = i >> 8, pair = i & 255;
            unsigned out = 0;
            if (valid(r))
            {
                const int j = row0 + r;
                const unsigned c = reinterpret_cast<const unsigned*>(a.cond + static_cast<size_t>(a.lane_rows[j]) * 512)[pair];
                const unsigned p = reinterpret_cast<const unsigned*>(a.positions + a.books[j] * 512)[pair];
                out = static_cast<unsigned>(add_bf16(c & 0xffffu, p & 0xffffu)) |
                      (static_cast<unsigned>(add_bf16(c >> 16, p >> 16)) << 16);
            }
            reinterpret_cast<unsigned*>(sh.h[r])[pair] = out;
        }
        __syncthreads();
    }
    else
    {
        // Feedback embedding sum over the earlier books (embed_sum_kernel's order).
        for (int i = tid; i < R * 128; i += THREADS)
        {
            const int r = i >> 7, c0 = (i & 127) * 8;
            std::uint16_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (valid(r))
            {
                const int j = row0 + r;
                const int count = a.counts[j];
                for (int e = 0; e < count; ++e)
                {
                    const int token = a.tokens[a.offsets[j] + e] & 1023;
                    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(
                        a.embeddings + (static_cast<size_t>(e) * 1024 + token) * 1024 + c0));
                    const std::uint16_t* v = reinterpret_cast<const std::uint16_t*>(&raw);
#pragma unroll
                    for (int x = 0; x < 8; ++x)
                        acc[x] = e == 0 ? v[x] : add_bf16(acc[x], v[x]);
                }
            }
            *reinterpret_cast<uint4*>(&sh.stage[r][c0]) = *reinterpret_cast<const uint4*>(acc);
        }
        __syncthreads();
        quantize_rows(4, [&](int r, int b, int l)
                      { return *reinterpret_cast<const uint4*>(&sh.stage[r][b * 256 + l * 8]); });
        __syncthreads();
        cta_linear(a.proj61, 512, 1024, 8, [&](int i) { return rank * 128 + i * 16; }, sh, ring_uses, timed_out,
                   [&](int m, int n, float s)
                   {
                       std::uint16_t y = to_bf16(__fadd_rn(s, __ldg(a.proj61.bias + n)));
                       if (valid(m))
                           y = add_bf16(y, a.positions[a.books[row0 + m] * 512 + n]);
                       sh.h_slice[m][n - rank * 128] = y;
                   });
        cluster.sync();
        gather_h();
        __syncthreads();
    }

    // ------------------------------------------------------------ layers --
    for (int l = 0; l < 3; ++l)
    {
        std::uint16_t* ck = a.cache_k + a.cache_stride * static_cast<size_t>(l);
        std::uint16_t* cv = a.cache_v + a.cache_stride * static_cast<size_t>(l);
        layer_norm_rows(2 * l);
        __syncthreads();
        // QKV of head `rank`: tiles 0-7 q, 8-15 k, 16-23 v.
        cta_linear(a.layer[l][0], 1536, 512, 24,
                   [&](int i) { return (i >> 3) * 512 + rank * 128 + (i & 7) * 16; }, sh, ring_uses, timed_out,
                   [&](int m, int n, float s)
                   {
                       const std::uint16_t y = to_bf16(__fadd_rn(s, __ldg(a.layer[l][0].bias + n)));
                       const int col = (n & 511) - rank * 128;
                       if (n < 512)
                           sh.q_head[m][col] = y;
                       else if (valid(m))
                       {
                           const size_t at = static_cast<size_t>(a.meta[row0 + m].slot) * 512 + (n & 511);
                           (n < 1024 ? ck : cv)[at] = y;
                       }
                   });
        __syncthreads();
        {
            const int group = tid >> 7, t = tid & 127;
            for (int r = group; r < R; r += 2)
            {
                std::uint16_t out = 0;
                if (valid(r))
                {
                    const RowMeta m = a.meta[row0 + r];
                    const AttentionBlock b =
                        attention_block_core(sh.q_head[r], m, rank, ck, cv, 0, m.time, sh.att[group], 1 + group, t);
                    out = attention_single_output(b);
                }
                sh.att_out[r][t] = out;
            }
        }
        cluster.sync();
        // Attention outputs of the four heads: 256-block b = heads 2b, 2b+1.
        quantize_rows(2, [&](int r, int b, int ln)
                      {
                          const int head = 2 * b + (ln >> 4);
                          return *reinterpret_cast<const uint4*>(&peer[head]->att_out[r][(ln & 15) * 8]);
                      });
        __syncthreads();
        cta_linear(a.layer[l][1], 512, 512, 8, [&](int i) { return rank * 128 + i * 16; }, sh, ring_uses, timed_out,
                   [&](int m, int n, float s)
                   {
                       const std::uint16_t y = to_bf16(__fadd_rn(s, __ldg(a.layer[l][1].bias + n)));
                       sh.h_slice[m][n - rank * 128] = add_bf16(sh.h[m][n], y);
                   });
        cluster.sync();
        gather_h();
        __syncthreads();
        layer_norm_rows(2 * l + 1);
        __syncthreads();
        cta_linear(a.layer[l][2], 2048, 512, 32, [&](int i) { return rank * 512 + i * 16; }, sh, ring_uses, timed_out,
                   [&](int m, int n, float s)
                   {
                       const std::uint16_t y = to_bf16(__fadd_rn(s, __ldg(a.layer[l][2].bias + n)));
                       sh.stage[m][n - rank * 512] = a.gelu[y];
                   });
        __syncthreads();
        // BF8L of this CTA's two 256-blocks of the FFN-in row.
        for (int task = warp; task < R * 2; task += THREADS / 32)
        {
            const int r = task >> 1, b = task & 1;
            bool ok = true;
            const Bf8lLane q = bf8l_block(*reinterpret_cast<const uint4*>(&sh.stage[r][b * 256 + lane * 8]), ok);
            finite = finite && (ok || !valid(r));
            *reinterpret_cast<uint2*>(&sh.mlp_q[r][b * 256 + lane * 8]) = make_uint2(q.packed[0], q.packed[1]);
            if (lane == 0)
                sh.mlp_s[r][b] = q.scale;
        }
        cluster.sync();
        for (int i = tid; i < R * 128; i += THREADS) // 16-byte pieces of the 2048-wide rows
        {
            const int r = i >> 7, piece = i & 127, owner = piece >> 5;
            *reinterpret_cast<uint4*>(&sh.xq[r][piece * 16]) =
                *reinterpret_cast<const uint4*>(&peer[owner]->mlp_q[r][(piece & 31) * 16]);
        }
        if (tid < R * 8)
        {
            const int r = tid >> 3, b = tid & 7;
            sh.xs[r][b] = peer[b >> 1]->mlp_s[r][b & 1];
        }
        __syncthreads();
        cta_linear(a.layer[l][3], 512, 2048, 8, [&](int i) { return rank * 128 + i * 16; }, sh, ring_uses, timed_out,
                   [&](int m, int n, float s)
                   {
                       const std::uint16_t y = to_bf16(__fadd_rn(s, __ldg(a.layer[l][3].bias + n)));
                       sh.h_slice[m][n - rank * 128] = add_bf16(sh.h[m][n], y);
                   });
        cluster.sync();
        gather_h();
        __syncthreads();
    }

    // ------------------------------------------------------------ output --
    layer_norm_rows(6);
    __syncthreads();
    cta_linear(a.proj62, 1024, 512, 16, [&](int i) { return rank * 256 + i * 16; }, sh, ring_uses, timed_out,
               [&](int m, int n, float s)
               { sh.logit_slice[m][n - rank * 256] = to_bf16(__fadd_rn(s, __ldg(a.proj62.bias + n))); });
    cluster.sync();
    for (int r = rank; r < R; r += CL)
    {
        if (!valid(r)) // uniform across the CTA
            continue;
        for (int i = tid; i < 128; i += THREADS) // 16-byte pieces of the 1024-wide row
            *reinterpret_cast<uint4*>(&sh.stage[0][i * 8]) =
                *reinterpret_cast<const uint4*>(&peer[i >> 5]->logit_slice[r][(i & 31) * 8]);
        __syncthreads();
        const bool ok = softmax_tree_row(sh.stage[0], nullptr, nullptr,
                                         a.tree + static_cast<size_t>(row0 + r) * 1023, sh.soft);
        finite = finite && ok;
    }
    if (!finite && a.error_word)
        atomicOr(a.error_word, error_nonfinite);
    if (timed_out && a.error_word)
        atomicOr(a.error_word, error_timeout);
    // Peers may still read this CTA's shared memory until every CTA is here.
    cluster.sync();
}
} // namespace

void codebook_step(const CodebookStepArgs& args, cudaStream_t stream)
{
    if (args.rows <= 0)
        return;
    constexpr size_t smem = sizeof(StepShared);
    static std::once_flag attr_once[64];
    int device = 0;
    cudaGetDevice(&device);
    if (device >= 0 && device < 64)
        std::call_once(attr_once[device],
                       []
                       {
                           cudaFuncSetAttribute(codebook_step_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem));
                       });
    const int clusters = (args.rows + R - 1) / R;
    codebook_step_kernel<<<clusters * CL, THREADS, smem, stream>>>(args);
    note_launch();
}
} // namespace tsacb::dev
