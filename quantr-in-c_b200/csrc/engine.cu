// engine.cu -- persistent, warp-specialized quantized-GEMV engine (sm_100a).
//
// One launch executes a "program": a list of independent GEMV jobs
// (out_j = W_j . x_j for B_j tokens).  Each job's rows are cut into tiles of
// R_j rows; the (job, tile) items are dealt round-robin to one persistent CTA
// per SM.  Inside a CTA three warp roles form a pipeline:
//
//   producer (1 warp)    streams each item's packed weight rows (one
//                        contiguous, 16-byte aligned range) and the job's
//                        quantized activations into a ring of S shared-memory
//                        slots with cp.async.bulk, plus a small item header;
//                        mbarrier transaction counts signal "slot full".  It
//                        runs up to S items ahead, so HBM streaming never waits
//                        for compute.
//   consumers (16 warps) decode one row x super-block (or Q8_0 block) per
//                        thread and evaluate the reference's exact per-unit
//                        terms (dp4a integer sums, explicitly rounded fp32
//                        ops) into one of T term buffers.  Work is dealt
//                        round-robin over the concatenation of all items, so a
//                        thread idle at the end of one tile starts the next.
//   chain (3 warps)      sum each (row, token)'s terms left to right - the
//                        reference's accumulation order, src/quant.c:279-285,
//                        :384-401, :422-435 - and store the fp32 outputs,
//                        while the consumers already work on later items.
//
// All waits are bounded (250 ms) and a CTA-wide abort flag stops every role if
// one of them gives up; slots with copies in flight are drained (bounded)
// before the CTA exits.  No multicast is used.  The quantized activations of
// every job are produced by k_quant_tasks (one launch per program run, the
// reference's quantize_row_q8_0 per input) in the compact, weight-type
// permuted layout the consumers read; the program kernel issues its first
// weight copies before griddepcontrol.wait, so under programmatic dependent
// launch the weight stream overlaps the quantizer.  Each launch runs a kernel
// built for its weight type when all jobs share one, for one-token jobs and
// for the row-fastest work order (smaller code: fewer instruction-fetch
// stalls).
#include "quantr_cuda.h"

#include "device_common.cuh"
#include "engine_act.cuh"
#include "formats.cuh"
#include "kernels.cuh"
#include "launch_util.cuh"
#include "libm_ref.cuh"
#include "quant_decode.cuh"

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <numeric>
#include <tuple>
#include <vector>

namespace qr {
namespace eng {

#ifndef QR_ENG_CONSUMER_WARPS
#define QR_ENG_CONSUMER_WARPS 16
#endif
#ifndef QR_ENG_CHAIN_WARPS
#define QR_ENG_CHAIN_WARPS 3
#endif
constexpr int kConsumerWarps = QR_ENG_CONSUMER_WARPS;
constexpr int kChainWarps = QR_ENG_CHAIN_WARPS;
constexpr int kWarps = 1 + kConsumerWarps + kChainWarps;
constexpr int kThreads = 32 * kWarps;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
// Ring depths: 3 weight slots of ~44 KB measured best on B200 for the c2
// shapes (fewer, larger tiles amortise the per-tile hand-off across the 12
// consumer warps; 3 x 44 KB in flight per SM still saturates HBM).
#ifndef QR_ENG_SLOTS
#define QR_ENG_SLOTS 3
#endif
#ifndef QR_ENG_SLOT_KB
#define QR_ENG_SLOT_KB 44
#endif
// Longest suspension (ns) of one barrier poll: a waiting warp sleeps until
// the phase completes (or this long) instead of spinning on issue slots the
// working warps need.
#ifndef QR_ENG_SUSPEND_NS
#define QR_ENG_SUSPEND_NS 1000
#endif
constexpr unsigned kSuspendNs = QR_ENG_SUSPEND_NS;
#ifndef QR_ENG_TERMS
#define QR_ENG_TERMS 4
#endif
// Tile shrinking: a launch with fewer than QR_ENG_MIN_ITEMS_PCT / 100 items
// per SM halves its tiles until it has that many.  Off by default: for the
// small one-token programs of a decode step (2.4-13 MB of weights each) fewer,
// larger items measured faster on B200 - the c3 step took 1.481 ms per token
// at 2 items per SM, 1.331 at 1, 1.268 at 0.5 and 1.244 with no shrinking.
// (A probable reason: a small launch then leaves SMs free, where the next
// kernel of the step is resident before this one completes.)
#ifndef QR_ENG_MIN_ITEMS_PCT
#define QR_ENG_MIN_ITEMS_PCT 0
#endif
constexpr int kMaxS = QR_ENG_SLOTS, kMaxT = QR_ENG_TERMS;
constexpr int kMaxB = 16;
constexpr size_t kSmemMax = 227 * 1024;
constexpr uint32_t kBulkChunk = 32768;
constexpr uint32_t kHdr = 128;  // bytes reserved for the item header in slots and term buffers

// Device-side job description (built by the host planner).
// Item header the producer writes at the start of a slot (and the consumers
// forward to the chain in the term buffer).
// 16-byte aligned: headers are copied with 128-bit loads/stores, including
// from a job passed inline in the kernel parameters.
struct __align__(16) ItemHdr {
    float* out;  // first output row of the tile
    long long ldo;
    uint32_t type, rb, nblk, B, U, TS, ds_off, rows, gfast;
    float inv_rows;             // 1/rows (approximate; only seeds an exact divmod)
    unsigned long long magic;   // floor(i / nblk) == (i * magic) >> 40
};
static_assert(sizeof(ItemHdr) == 64, "item header is copied as four 16-byte words");

struct __align__(16) JobDesc {
    ItemHdr hdr;         // template of every tile's header (out = job base, rows = R)
    const uint8_t* w;    // 16-byte aligned packed rows
    const uint8_t* act;  // quantized activations: q[B][U][32] | ds[B][U] (fp32 scale, quant sum as fp32)
    long long rb;
    uint32_t act_bytes;
    int n, U, R, tiles, item0, pad_[4];
};
static_assert(sizeof(JobDesc) % 16 == 0, "job table is copied in 16-byte words");

// Jobs per engine launch: the launch keeps its job table in shared memory
// (read by the producer for every item; global reads would sit behind the
// weight stream in L2).  Larger programs are split into several launches.
constexpr int kMaxJobsPerLaunch = 96;

static_assert(sizeof(ItemHdr) <= kHdr, "item header too large");

struct ProgParams {
    const JobDesc* jobs;  // null: use inline_job
    int njobs, total_items;
    uint32_t slot_bytes, slot_x_off, term_bytes, S, T;
    uint32_t slot_off, term_off, jobs_off;
    int* err;
    JobDesc inline_job;
};
static_assert(offsetof(ProgParams, inline_job) % 16 == 0, "inline job must be 16-byte aligned in param space");

// One quantization task: B rows of fp32 x -> the compact act layout.
struct QTask {
    const float* x;
    const float* xmul;  // non-null: the input is silu(x) * xmul, elementwise
    uint8_t* act;
    long long ldx;
    long long blk0;  // first global block index of this task
    int U, B, type;
    uint32_t ds_off;
};

struct QParams {
    const QTask* tasks;  // null: use inline_task
    int ntasks;
    long long total_blocks;
    QTask inline_task;
};


// Integer -> float conversions of the consumers.  Every converted value is an
// integer of magnitude below 2^22, so adding it to the bit pattern of
// 1.5 * 2^23 (whose ulp is 1) and subtracting 1.5 * 2^23 in fp32 gives the
// same float as a conversion, exactly, on the full-rate add pipe.  The
// activation records carry the block's quant sum as a float for the same
// reason (|sum| <= 32 * 127).
constexpr int kCvtBias = 0x4B400000;
constexpr float kCvtBiasF = 12582912.0f;
// float(v) for 0 <= v < 2^23 (scale codes)
__device__ __forceinline__ float small_u2f(uint32_t v) { return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.0f); }

// Reference quantize_row_q8_0 (src/quant.c:143-158), one warp per block,
// writing the engine's compact layout for the consuming job's weight type.
constexpr int kMaxTasksInSmem = 256;

__global__ void __launch_bounds__(256) k_quant_tasks(const __grid_constant__ QParams p)
{
    // The task table (written by the host at program creation) is searched
    // once per block of 32 elements: keep it in shared memory.
    __shared__ QTask stasks[kMaxTasksInSmem];
    const QTask* tasks = p.tasks ? p.tasks : &p.inline_task;
    if (p.tasks && p.ntasks <= kMaxTasksInSmem) {
        for (int t = threadIdx.x; t < p.ntasks; t += blockDim.x) stasks[t] = p.tasks[t];
        __syncthreads();
        tasks = stasks;
    }
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long step = (long long)gridDim.x * 8;
    for (long long gb = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); gb < p.total_blocks; gb += step) {
        int lo = 0, hi = p.ntasks - 1;  // last task with blk0 <= gb
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (tasks[mid].blk0 <= gb) lo = mid; else hi = mid - 1;
        }
        const QTask& T = tasks[lo];
        const long long local = gb - T.blk0;
        const int t = (int)(local / T.U), b = (int)(local - (long long)t * T.U);
        const long long xi = (long long)t * T.ldx + (long long)b * 32 + lane;
        const float v = T.xmul ? libm::swiglu_ref(T.x[xi], T.xmul[xi]) : T.x[xi];
        act_write_block(T.act, T.ds_off, T.U, T.type, t, b, lane, v);
    }
}

__device__ __forceinline__ int job_of(const JobDesc* jobs, int njobs, int item, int jc)
{
    while (jc + 1 < njobs && item >= jobs[jc + 1].item0) ++jc;
    return jc;
}

// ------------------------------------------------------------ consumers --
//
// All shared-memory accesses below are `sm + 32-bit offset` with `sm` the
// kernel's __shared__ base, so they compile to shared-window loads/stores.

// Per-item values, read from the item header into registers once per item.
struct Item {
    uint32_t tile;   // offset of the weight tile
    uint32_t xq;     // offset of q[B][U][32]
    uint32_t ds;     // offset of ds[B][U] (8 bytes each)
    uint32_t terms;  // offset of terms[U][TS]
    int rb, nblk, B, U, TS;
};

template <bool ONE, int KIND>
__device__ __forceinline__ void put_terms(uint8_t* sm, const Item& it, int g, int tu, int xu, float a, float b,
                                          const uint32_t (&wq)[8])
{
    const int nb = ONE ? 1 : it.B;
    for (int t = 0; t < nb; ++t) {
        const uint32_t xo = it.xq + (uint32_t)((t * it.U + xu) * 32);
        const uint4 xa = *reinterpret_cast<const uint4*>(sm + xo);
        const uint4 xb = *reinterpret_cast<const uint4*>(sm + xo + 16);
        const uint2 ds = *reinterpret_cast<const uint2*>(sm + it.ds + (uint32_t)((t * it.U + xu) * 8));
        const float dx = __uint_as_float(ds.x);
        float term;
        // The reference's term (src/quant.c:284, :433, :399) on exactly converted operands.
        const float isf = __fsub_rn(__int_as_float(dot8_from(wq, xa, xb, kCvtBias)), kCvtBiasF);
        const float bsf = __uint_as_float(ds.y);
        if (KIND == 0) term = __fmul_rn(__fmul_rn(isf, a), dx);
        else if (KIND == 2) term = __fmul_rn(__fmul_rn(a, __fsub_rn(isf, __fmul_rn(32.0f, bsf))), dx);
        else term = __fmul_rn(__fsub_rn(__fmul_rn(a, isf), __fmul_rn(b, bsf)), dx);
        *reinterpret_cast<float*>(sm + it.terms + (uint32_t)((tu * it.TS + g * nb + t) * 4)) = term;
    }
}

// Q4_K / Q5_K super-block (16-byte aligned): header and quants by 128-bit
// loads.  Q4_K keeps the high nibble in place and divides its dp4a product
// by 16 (exact: every product is a multiple of 16).
template <uint32_t TYPE, bool ONE>
__device__ __forceinline__ void consume_k45(uint8_t* sm, const Item& it, int g, int s)
{
    const uint32_t sb = it.tile + (uint32_t)(g * it.rb + s * block_bytes(TYPE));
    const uint4 hdr = *reinterpret_cast<const uint4*>(sm + sb);
    const float d = h2f_ref(hdr.x & 0xFFFFu), dmin = h2f_ref(hdr.x >> 16);
    uint4 qh0 = make_uint4(0, 0, 0, 0), qh1 = qh0;
    if (TYPE == T_Q5_K) {
        qh0 = *reinterpret_cast<const uint4*>(sm + sb + 16);
        qh1 = *reinterpret_cast<const uint4*>(sm + sb + 32);
    }
    const uint32_t qs = sb + (TYPE == T_Q4_K ? 16u : 48u);
    const int nb = ONE ? 1 : it.B;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t scb = ((j < 4 ? hdr.y : hdr.z) >> (8 * (j & 3))) & 0xFFu;
        const float sc = __fmul_rn(small_u2f(scb & 63u), d);    // src/quant.c:385
        const float m = __fmul_rn(small_u2f(scb >> 6), dmin);   // src/quant.c:386
        const uint4 q = *reinterpret_cast<const uint4*>(sm + qs + 16 * j);
        const int tu = 8 * s + j, xu = j * it.nblk + s;
        if (TYPE == T_Q4_K) {
            const uint32_t l0 = q.x & 0x0F0F0F0Fu, l1 = q.y & 0x0F0F0F0Fu, l2 = q.z & 0x0F0F0F0Fu,
                           l3 = q.w & 0x0F0F0F0Fu;
            const uint32_t h0 = q.x & 0xF0F0F0F0u, h1 = q.y & 0xF0F0F0F0u, h2 = q.z & 0xF0F0F0F0u,
                           h3 = q.w & 0xF0F0F0F0u;
            for (int t = 0; t < nb; ++t) {
                const uint32_t xo = it.xq + (uint32_t)((t * it.U + xu) * 32);
                const uint4 xa = *reinterpret_cast<const uint4*>(sm + xo);
                const uint4 xb = *reinterpret_cast<const uint4*>(sm + xo + 16);
                const uint2 ds = *reinterpret_cast<const uint2*>(sm + it.ds + (uint32_t)((t * it.U + xu) * 8));
                int lo = __dp4a((int)l0, (int)xa.x, kCvtBias);
                lo = __dp4a((int)l1, (int)xa.z, lo);
                lo = __dp4a((int)l2, (int)xb.x, lo);
                lo = __dp4a((int)l3, (int)xb.z, lo);
                int hi = dp4a_us(h0, (int)xa.y, 0);
                hi = dp4a_us(h1, (int)xa.w, hi);
                hi = dp4a_us(h2, (int)xb.y, hi);
                hi = dp4a_us(h3, (int)xb.w, hi);
                const int isum = lo + (hi >> 4);
                // src/quant.c:399 on exactly converted operands
                const float term = __fmul_rn(__fsub_rn(__fmul_rn(sc, __fsub_rn(__int_as_float(isum), kCvtBiasF)),
                                                       __fmul_rn(m, __uint_as_float(ds.y))),
                                             __uint_as_float(ds.x));
                *reinterpret_cast<float*>(sm + it.terms + (uint32_t)((tu * it.TS + g * nb + t) * 4)) = term;
            }
        } else {
            const uint32_t H = (j < 4) ? (j == 0 ? qh0.x : j == 1 ? qh0.y : j == 2 ? qh0.z : qh0.w)
                                       : (j == 4 ? qh1.x : j == 5 ? qh1.y : j == 6 ? qh1.z : qh1.w);
            uint32_t wq[8];
            const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t hb = (H >> (8 * i)) & 0xFFu;
                wq[2 * i] = (qw[i] & 0x0F0F0F0Fu) | spread_even_bits_to_b4(hb);
                wq[2 * i + 1] = ((qw[i] >> 4) & 0x0F0F0F0Fu) | spread_even_bits_to_b4(hb >> 1);
            }
            put_terms<ONE, 1>(sm, it, g, tu, xu, sc, m, wq);
        }
    }
}

// Q6_K super-block (2-byte aligned: 210-byte blocks) by funnel-shifted words.
template <bool ONE>
__device__ __forceinline__ void consume_q6k(uint8_t* sm, const Item& it, int g, int s)
{
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sm);
    const uint32_t sb = it.tile + (uint32_t)(g * it.rb) + 210u * (uint32_t)s;
    uint32_t scw[2];
    ld_words<2>(s32, sb + 192, scw);
    const float d = h2f_ref(ld_u32(s32, sb + 208) & 0xFFFFu);
#pragma unroll 2
    for (int j = 0; j < 8; ++j) {
        const float sc = __fmul_rn((float)(int8_t)((scw[j >> 2] >> (8 * (j & 3))) & 0xFFu), d);  // :423
        uint32_t ql[4], qh[2], wq[8];
        ld_words<4>(s32, sb + 16u * j, ql);
        ld_words<2>(s32, sb + 128u + 8u * j, qh);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t s0 = __byte_perm(ql[2 * h], ql[2 * h + 1], 0x6420);
            const uint32_t s1 = __byte_perm(ql[2 * h], ql[2 * h + 1], 0x7531);
            const uint32_t nib[4] = {s0 & 0x0F0F0F0Fu, (s0 >> 4) & 0x0F0F0F0Fu, s1 & 0x0F0F0F0Fu,
                                     (s1 >> 4) & 0x0F0F0F0Fu};
#pragma unroll
            for (int m = 0; m < 4; ++m) wq[4 * h + m] = nib[m] | (((qh[h] >> (2 * m)) & 0x03030303u) << 4);
        }
        put_terms<ONE, 2>(sm, it, g, 8 * s + j, j * it.nblk + s, sc, 0.0f, wq);
    }
}

// Q8_0 block (34 bytes, 2-byte aligned).
template <bool ONE>
__device__ __forceinline__ void consume_q80(uint8_t* sm, const Item& it, int g, int u)
{
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sm);
    const uint32_t blk = it.tile + (uint32_t)(g * it.rb) + 34u * (uint32_t)u;
    const float dw = h2f_ref(ld_u32(s32, blk) & 0xFFFFu);
    uint32_t wq[8];
    ld_words<8>(s32, blk + 2, wq);
    put_terms<ONE, 0>(sm, it, g, u, u, dw, 0.0f, wq);
}

// Work index -> (row g, block s).  Block-fastest by default (neighbouring
// lanes read neighbouring blocks of one row).  Row-fastest (`gfast`) when the
// planner found the row stride an odd number of 16-byte units (Q4_K/Q5_K):
// a warp's lanes then share one super-block column, so activation reads are
// broadcasts and weight reads still hit distinct banks.
template <uint32_t TYPE, bool ONE>
__device__ __forceinline__ void consume_range(uint8_t* sm, const Item& it, int first, int total,
                                              unsigned long long magic, int rows, float inv_rows, bool gfast)
{
    for (int i = first; i < total; i += kConsumerThreads) {
        int g, s;
        if (gfast) {
            s = (int)((float)i * inv_rows);  // within one of the true quotient; corrected below
            g = i - s * rows;
            if (g < 0) { --s; g += rows; }
            else if (g >= rows) { ++s; g -= rows; }
        } else {
            g = (int)(((unsigned long long)i * magic) >> 40);
            s = i - g * it.nblk;
        }
        if (TYPE == T_Q4_K || TYPE == T_Q5_K) consume_k45<TYPE, ONE>(sm, it, g, s);
        else if (TYPE == T_Q6_K) consume_q6k<ONE>(sm, it, g, s);
        else consume_q80<ONE>(sm, it, g, s);
    }
}

template <uint32_t TYPE, bool ONE_ONLY, bool GFAST_ALL>
__device__ __forceinline__ void consume_typed(uint8_t* sm, const Item& it, int first, int total, const ItemHdr& h)
{
    const bool gfast = (TYPE == T_Q4_K || TYPE == T_Q5_K) && (GFAST_ALL || h.gfast);
    if (ONE_ONLY || it.B == 1) consume_range<TYPE, true>(sm, it, first, total, h.magic, (int)h.rows, h.inv_rows, gfast);
    else consume_range<TYPE, false>(sm, it, first, total, h.magic, (int)h.rows, h.inv_rows, gfast);
}

// ---------------------------------------------------------------- kernel --

// TY: the weight type every job of the launch shares (only its consumer code
// is built in), or -1 for launches that mix types; ONE: every job has one
// token (programs send wider jobs to the tensor cores); GF: every job takes
// the row-fastest work order.
template <int TY, bool ONE, bool GF>
__global__ void __launch_bounds__(kThreads, 1) k_program(const __grid_constant__ ProgParams p)
{
    extern __shared__ __align__(1024) uint8_t sm[];
    uint64_t* wfull = reinterpret_cast<uint64_t*>(sm);
    uint64_t* wempty = wfull + kMaxS;
    uint64_t* tfull = wempty + kMaxS;
    uint64_t* tempty = tfull + kMaxT;
    int* ctl = reinterpret_cast<int*>(tempty + kMaxT);  // [0] abort, [1..S] fills issued per slot
    volatile int* abort_flag = ctl;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int P = gridDim.x, c = blockIdx.x;
    const int S = (int)p.S, T = (int)p.T;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], kConsumerWarps);
            ctl[1 + s] = 0;
        }
        for (int t = 0; t < T; ++t) {
            mbar_init(&tfull[t], kConsumerWarps);
            mbar_init(&tempty[t], 1);
        }
        ctl[0] = 0;
        mbar_fence_init();
    }
    if (p.jobs) {  // job table -> shared memory (written by the host before any launch)
        const uint4* src = reinterpret_cast<const uint4*>(p.jobs);
        uint4* dst = reinterpret_cast<uint4*>(sm + p.jobs_off);
        const int words = p.njobs * (int)(sizeof(JobDesc) / 16);
        for (int w = threadIdx.x; w < words; w += kThreads) dst[w] = src[w];
    }
    __syncthreads();
    pdl_trigger();

    if (warp == 0) {
        // ------------------------------------------------------ producer --
        if (lane == 0) {
            const JobDesc* jobs = p.jobs ? reinterpret_cast<const JobDesc*>(sm + p.jobs_off) : &p.inline_job;
            int jc = 0, k = 0, i = c;
            int pend_job[kMaxS] = {};
            auto issue_w = [&](const JobDesc& J, int item, int slot) {
                const int r0 = (item - J.item0) * J.R;
                const int rows = min(J.R, J.n - r0);
                const uint8_t* src = J.w + (long long)r0 * J.rb;
                uint8_t* base = sm + p.slot_off + (size_t)slot * p.slot_bytes;
                // Header: the job's template, patched for this tile.
                const uint4* hs = reinterpret_cast<const uint4*>(&J.hdr);
                uint4* hd = reinterpret_cast<uint4*>(base);
                hd[0] = hs[0];
                hd[1] = hs[1];
                hd[2] = hs[2];
                hd[3] = hs[3];
                ItemHdr* h = reinterpret_cast<ItemHdr*>(base);
                if (r0) h->out = J.hdr.out + r0;
                if (rows != J.R) {
                    h->rows = (uint32_t)rows;
                    h->inv_rows = __frcp_rn((float)rows);
                }
                uint8_t* dst = base + kHdr;
                const uint32_t bytes = (uint32_t)(rows * J.rb);
                const uint32_t body = bytes & ~15u;
                for (uint32_t b = body; b < bytes; ++b) dst[b] = src[b];  // < 16 ragged bytes
                mbar_arrive_expect_tx(&wfull[slot], body + J.act_bytes);
                for (uint32_t off = 0; off < body; off += kBulkChunk)
                    bulk_g2s(dst + off, src + off, min(kBulkChunk, body - off), &wfull[slot]);
                ctl[1 + slot] += 1;
            };
            auto issue_x = [&](const JobDesc& J, int slot) {
                uint8_t* dst = sm + p.slot_off + (size_t)slot * p.slot_bytes + p.slot_x_off;
                bulk_g2s(dst, J.act, J.act_bytes, &wfull[slot]);
            };
            // Prologue: weights of the first S items before waiting for the
            // quantizer grid (weights never depend on it).
            for (; k < S && i < p.total_items; ++k, i += P) {
                jc = job_of(jobs, p.njobs, i, jc);
                issue_w(jobs[jc], i, k);
                pend_job[k] = jc;
            }
            pdl_wait();
            for (int q = 0; q < k; ++q) issue_x(jobs[pend_job[q]], q);
            for (; i < p.total_items; ++k, i += P) {
                jc = job_of(jobs, p.njobs, i, jc);
                const int slot = k % S;
                if (!mbar_wait_bounded(&wempty[slot], ((k / S) - 1) & 1, p.err, abort_flag, kSuspendNs)) break;
                issue_w(jobs[jc], i, slot);
                issue_x(jobs[jc], slot);
            }
        }
    } else if (warp <= kConsumerWarps) {
        // ----------------------------------------------------- consumers --
        const int ctid = (warp - 1) * 32 + lane;
        int rot = 0;  // sum of earlier items' work, mod kConsumerThreads
        for (int k = 0, i = c; i < p.total_items; ++k, i += P) {
            const int slot = k % S, tb = k % T;
            if (!mbar_wait_bounded(&wfull[slot], (k / S) & 1, p.err, abort_flag, kSuspendNs)) break;
            if (k >= T && !mbar_wait_bounded(&tempty[tb], ((k / T) - 1) & 1, p.err, abort_flag, kSuspendNs)) break;
            const uint32_t base = p.slot_off + (uint32_t)slot * p.slot_bytes;
            const ItemHdr h = *reinterpret_cast<const ItemHdr*>(sm + base);
            Item it;
            it.tile = base + kHdr;
            it.xq = base + p.slot_x_off;
            it.ds = it.xq + h.ds_off;
            it.terms = p.term_off + (uint32_t)tb * p.term_bytes + kHdr;
            it.rb = (int)h.rb;
            it.nblk = (int)h.nblk;
            it.B = (int)h.B;
            it.U = (int)h.U;
            it.TS = (int)h.TS;
            const int total = (int)h.rows * it.nblk;
            const int first = ctid >= rot ? ctid - rot : ctid - rot + kConsumerThreads;
            rot = (int)(((unsigned)rot + (unsigned)total) % (unsigned)kConsumerThreads);
            if constexpr (TY >= 0) {
                consume_typed<(uint32_t)TY, ONE, GF>(sm, it, first, total, h);
            } else {
                switch (h.type) {
                case T_Q4_K: consume_typed<T_Q4_K, ONE, false>(sm, it, first, total, h); break;
                case T_Q5_K: consume_typed<T_Q5_K, ONE, false>(sm, it, first, total, h); break;
                case T_Q6_K: consume_typed<T_Q6_K, ONE, false>(sm, it, first, total, h); break;
                default: consume_typed<T_Q8_0, ONE, false>(sm, it, first, total, h); break;
                }
            }
            if (ctid == 0)  // forward the header to the chain warps
                *reinterpret_cast<ItemHdr*>(sm + p.term_off + (uint32_t)tb * p.term_bytes) = h;
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tfull[tb]);
                mbar_arrive(&wempty[slot]);
            }
        }
    } else {
        // --------------------------------------------------------- chain --
        const int ch = warp - 1 - kConsumerWarps;
        for (int k = ch, i = c + ch * P; i < p.total_items; k += kChainWarps, i += kChainWarps * P) {
            const int tb = k % T;
            if (!mbar_wait_bounded(&tfull[tb], (k / T) & 1, p.err, abort_flag, kSuspendNs)) break;
            const uint32_t tbase = p.term_off + (uint32_t)tb * p.term_bytes;
            const ItemHdr h = *reinterpret_cast<const ItemHdr*>(sm + tbase);
            const float* terms = reinterpret_cast<const float*>(sm + tbase + kHdr);
            const int B = (int)h.B, U = (int)h.U, TS = (int)h.TS, rows = (int)h.rows;
            float* out = h.out;
            const long long ldo = h.ldo;
            for (int q = lane; q < rows * B; q += 32) {
                const int g = ONE ? q : q / B, t = ONE ? 0 : q - g * B;
                const float* tp = terms + q;
                float acc = 0.0f;
#pragma unroll 8
                for (int u = 0; u < U; ++u) acc = __fadd_rn(acc, tp[u * TS]);
                out[(long long)t * ldo + g] = acc;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[tb]);
        }
    }

    __syncthreads();
    if (*abort_flag && threadIdx.x == 0) {
        // Some role gave up: let every copy this CTA issued land (bounded)
        // before its shared memory is released.
        for (int s = 0; s < S; ++s)
            if (ctl[1 + s] > 0) mbar_wait_bounded(&wfull[s], (ctl[1 + s] - 1) & 1, nullptr);
    }
}

// ------------------------------------------------------------ host side --

int gcd_int(long long a, long long b) { return (int)std::gcd(a, b); }

unsigned long long magic40(int dvs) { return ((1ULL << 40) + (unsigned long long)dvs - 1) / (unsigned long long)dvs; }

// One engine launch: its jobs, tiling and shared-memory layout.
struct SubPlan {
    std::vector<JobDesc> jobs;
    ProgParams pp{};
    int grid = 0;
    size_t smem = 0;
    JobDesc* d_jobs = nullptr;  // device job table; null for a single inline job
    int ty = -1;                // the weight type all jobs share, -1 if mixed
    bool one = false;           // every job has one token
    bool gfast = false;         // every job takes the row-fastest work order
};

struct Plan {
    std::vector<QTask> tasks;
    long long total_blocks = 0;
    size_t act_total = 0;
    QParams qp{};
    std::vector<SubPlan> subs;
};

struct JobIn {
    const uint8_t* w;
    uint32_t type;
    int n, d, B;
    const float* x;
    long long ldx;
    float* out;
    long long ldo;
    const float* xmul = nullptr;  // input is silu(x) * xmul (same strides)
};

int units_of(uint32_t type, int d) { return (d / block_elems(type)) * block_units(type); }

// Activation region of one input: q[B][U][32] then 8-byte (scale, quant sum as fp32) pairs.
size_t act_ds_off(uint32_t type, int d, int B) { return (size_t)B * units_of(type, d) * 32; }
size_t act_bytes_for(uint32_t type, int d, int B)
{
    return act_ds_off(type, d, B) + (((size_t)B * units_of(type, d) * 8 + 15) & ~size_t(15));
}

// Tiles and shared-memory layout of one launch.  `table`: the launch keeps a
// job table in shared memory (otherwise its single job travels inline).
int layout_sub(SubPlan& sp, int sms, bool table)
{
    // Optional tile shrinking (QR_ENG_MIN_ITEMS_PCT, off by default).
    auto count_items = [&]() {
        long long t = 0;
        for (auto& J : sp.jobs) t += (J.n + J.R - 1) / J.R;
        return t;
    };
    for (int iter = 0; iter < 16 && 100 * count_items() < (long long)QR_ENG_MIN_ITEMS_PCT * sms; ++iter) {
        bool changed = false;
        for (auto& J : sp.jobs) {
            const int gR = 16 / gcd_int(J.rb, 16);
            const int nr = std::max(gR, ((J.R / 2) / gR) * gR);
            if (nr < J.R) {
                J.R = nr;
                changed = true;
            }
        }
        if (!changed) break;
    }
    size_t slot_w = 0, slot_x = 0, term = 0;
    int item = 0;
    for (auto& J : sp.jobs) {
        J.hdr.TS = (uint32_t)((J.R * (int)J.hdr.B) | 1);
        J.hdr.rows = (uint32_t)J.R;
        J.hdr.inv_rows = 1.0f / (float)J.R;
        J.tiles = (J.n + J.R - 1) / J.R;
        J.item0 = item;
        item += J.tiles;
        slot_w = std::max(slot_w, (size_t)((long long)J.R * J.rb));
        slot_x = std::max(slot_x, (size_t)J.act_bytes);
        term = std::max(term, (size_t)J.U * J.hdr.TS * 4);
    }
    auto up128 = [](size_t v) { return (v + 127) & ~size_t(127); };
    slot_w = up128(slot_w);
    slot_x = up128(slot_x);
    term = kHdr + up128(term);
    const size_t slot = kHdr + slot_w + slot_x;
    const size_t bars = 1024;
    const size_t tbl = table ? up128(sp.jobs.size() * sizeof(JobDesc)) : 0;
    int T = kMaxT, S = 0;
    for (; T >= 3; --T) {
        if (bars + tbl + (size_t)T * term >= kSmemMax) continue;
        S = (int)std::min<size_t>(kMaxS, (kSmemMax - bars - tbl - (size_t)T * term) / slot);
        if (S >= 2) break;
    }
    if (S < 2) return QUANTR_ERR_TOO_LARGE;
    ProgParams& pp = sp.pp;
    pp.njobs = (int)sp.jobs.size();
    pp.total_items = item;
    pp.slot_bytes = (uint32_t)slot;
    pp.slot_x_off = (uint32_t)(kHdr + slot_w);
    pp.term_bytes = (uint32_t)term;
    pp.S = (uint32_t)S;
    pp.T = (uint32_t)T;
    pp.slot_off = (uint32_t)bars;
    pp.term_off = (uint32_t)(bars + (size_t)S * slot);
    pp.jobs_off = pp.term_off + (uint32_t)((size_t)T * term);
    sp.smem = pp.jobs_off + tbl;
    sp.grid = std::min(sms, item);
    return QUANTR_OK;
}

// Validates the jobs and lays out tiles, activations and shared memory.
// act_base == nullptr plans the sizes only.
// `tables`: every launch reads a device job table copied into shared memory
// (programs); false only for a single job passed inline (single-GEMV calls).
int make_plan(const JobIn* in, int njobs, uint8_t* act_base, int sms, bool tables, Plan& pl)
{
    pl = Plan{};
    if (njobs <= 0) return QUANTR_ERR_BAD_ARG;
    std::map<std::tuple<const float*, const float*, long long, int, int, int, int>, int> dedupe;  // x,xmul,ldx,d,B,U,perm
    constexpr size_t kSlotW = QR_ENG_SLOT_KB * 1024, kTermMax = 16 * 1024;
    std::vector<JobDesc> all;
    for (int j = 0; j < njobs; ++j) {
        const JobIn& a = in[j];
        if (!type_supported(a.type)) return QUANTR_ERR_UNSUPPORTED_TYPE;
        if (!a.w || !a.x || !a.out || a.n <= 0 || a.B <= 0 || a.B > kMaxB || a.ldx < a.d || a.ldo < a.n)
            return QUANTR_ERR_BAD_ARG;
        if (((uintptr_t)a.w & 15) != 0) return QUANTR_ERR_BAD_ARG;
        const long long rb = row_bytes(a.type, a.d);
        if (rb <= 0) return QUANTR_ERR_BAD_ARG;
        JobDesc J{};
        J.w = a.w;
        J.rb = rb;
        J.n = a.n;
        J.U = units_of(a.type, a.d);
        ItemHdr& H = J.hdr;
        H.out = a.out;
        H.ldo = a.ldo;
        H.type = a.type;
        H.rb = (uint32_t)rb;
        H.B = (uint32_t)a.B;
        H.U = (uint32_t)J.U;
        H.nblk = (uint32_t)(a.type == T_Q8_0 ? J.U : J.U / 8);
        H.magic = magic40((int)H.nblk);
        // Row-fastest work order for 16-byte aligned super-blocks whose row
        // stride is an odd number of 16-byte units (conflict-free rows).
        H.gfast = (a.type == T_Q4_K || a.type == T_Q5_K) && ((rb / 16) & 1) ? 1u : 0u;
        const int gR = 16 / gcd_int(rb, 16);  // R*rb % 16 == 0 keeps every tile 16-byte aligned
        auto round_dn = [&](long long v) { return std::max<long long>(gR, (v / gR) * gR); };
        long long R = round_dn((long long)(kSlotW / rb));
        const long long Rt = round_dn((long long)((kTermMax / (4 * (size_t)J.U) - 1) / a.B));
        R = std::min(R, Rt);
        R = std::min<long long>(R, ((a.n + gR - 1) / gR) * gR);
        J.R = (int)R;
        const int perm = a.type == T_Q8_0 ? 0 : (a.type == T_Q6_K ? 2 : 1);
        auto key = std::make_tuple(a.x, a.xmul, a.ldx, a.d, a.B, J.U, perm);
        auto it = dedupe.find(key);
        int ti;
        if (it == dedupe.end()) {
            QTask t{};
            t.x = a.x;
            t.xmul = a.xmul;
            t.ldx = a.ldx;
            t.U = J.U;
            t.B = a.B;
            t.type = (int)a.type;
            t.ds_off = (uint32_t)act_ds_off(a.type, a.d, a.B);
            t.blk0 = pl.total_blocks;
            t.act = act_base ? act_base + pl.act_total : nullptr;
            pl.total_blocks += (long long)a.B * J.U;
            pl.act_total += (act_bytes_for(a.type, a.d, a.B) + 255) & ~size_t(255);
            ti = (int)pl.tasks.size();
            pl.tasks.push_back(t);
            dedupe[key] = ti;
        } else {
            ti = it->second;
        }
        J.act = pl.tasks[ti].act;
        H.ds_off = pl.tasks[ti].ds_off;
        J.act_bytes = (uint32_t)act_bytes_for(a.type, a.d, a.B);
        all.push_back(J);
    }
    for (int j0 = 0; j0 < njobs; j0 += kMaxJobsPerLaunch) {
        SubPlan sp;
        sp.jobs.assign(all.begin() + j0, all.begin() + std::min(njobs, j0 + kMaxJobsPerLaunch));
        if (!tables && sp.jobs.size() != 1) return QUANTR_ERR_BAD_ARG;
        const int rc = layout_sub(sp, sms, tables);
        if (rc) return rc;
        sp.ty = (int)sp.jobs[0].hdr.type;
        sp.one = sp.gfast = true;
        for (const auto& J : sp.jobs) {
            if ((int)J.hdr.type != sp.ty) sp.ty = -1;
            if (J.hdr.B != 1) sp.one = false;
            if (!J.hdr.gfast) sp.gfast = false;
        }
        pl.subs.push_back(std::move(sp));
    }
    pl.qp.ntasks = (int)pl.tasks.size();
    pl.qp.total_blocks = pl.total_blocks;
    return QUANTR_OK;
}

template <int TY, bool ONE, bool GF>
cudaError_t launch_program_k(const SubPlan& sp, const ProgParams& pp, const LaunchCfg& c)
{
    static int configured_dev = -1;
    cudaError_t e = ensure_smem_attr(&k_program<TY, ONE, GF>, (int)kSmemMax, configured_dev);
    if (e != cudaSuccess) return e;
    return launch_ex(&k_program<TY, ONE, GF>, dim3(sp.grid), dim3(kThreads), sp.smem, c, pp);
}

template <int TY>
cudaError_t launch_program_t(const SubPlan& sp, const ProgParams& pp, const LaunchCfg& c)
{
    if constexpr (TY == T_Q4_K || TY == T_Q5_K) {  // the row-fastest order applies to these
        if (sp.one && sp.gfast) return launch_program_k<TY, true, true>(sp, pp, c);
    }
    return sp.one ? launch_program_k<TY, true, false>(sp, pp, c) : launch_program_k<TY, false, false>(sp, pp, c);
}

cudaError_t launch_program(const SubPlan& sp, const ProgParams& pp, const LaunchCfg& c)
{
    switch (sp.ty) {
    case T_Q4_K: return launch_program_t<T_Q4_K>(sp, pp, c);
    case T_Q5_K: return launch_program_t<T_Q5_K>(sp, pp, c);
    case T_Q6_K: return launch_program_t<T_Q6_K>(sp, pp, c);
    case T_Q8_0: return launch_program_t<T_Q8_0>(sp, pp, c);
    default: return launch_program_t<-1>(sp, pp, c);
    }
}

// Launches the quantizer over every task, then one engine launch per
// sub-plan (a single job travels inline when the sub-plan has no table).
cudaError_t launch_plan(Plan& pl, const QTask* d_tasks, int* err, cudaStream_t stream, bool skip_quant = false)
{
    LaunchCfg c;
    c.stream = stream;
    cudaError_t e = cudaSuccess;
    QParams qp = pl.qp;
    qp.tasks = d_tasks;
    if (!d_tasks) qp.inline_task = pl.tasks[0];
    const long long qgrid = std::max(1LL, std::min<long long>((qp.total_blocks + 7) / 8, 8LL * device_sm_count()));
    if (!skip_quant) e = launch_ex(&k_quant_tasks, dim3((unsigned)qgrid), dim3(256), 0, c, qp);
    for (auto& sp : pl.subs) {
        if (e != cudaSuccess) return e;
        ProgParams pp = sp.pp;
        pp.jobs = sp.d_jobs;
        if (!sp.d_jobs) pp.inline_job = sp.jobs[0];
        pp.err = err;
        e = launch_program(sp, pp, c);
    }
    return e;
}

} // namespace eng

// Single GEMV through the engine (no allocation: activations go to `ws`).
// Returns cudaErrorNotSupported when the engine cannot take this shape, so the
// caller can use the general kernel instead.
cudaError_t launch_gemv_engine(const uint8_t* w, uint32_t type, int n, int d, int B, const float* x, long long ldx,
                               float* out, long long ldo, void* ws, size_t ws_bytes, int* err, cudaStream_t stream)
{
    if (!type_supported(type) || ((uintptr_t)w & 15) || ((uintptr_t)ws & 15) || B > eng::kMaxB ||
        row_bytes(type, d) <= 0)
        return cudaErrorNotSupported;
    if (eng::act_bytes_for(type, d, B) > ws_bytes) return cudaErrorNotSupported;
    // Plans depend only on these arguments and the device; repeated calls
    // (a decoder's per-layer GEMVs) reuse them instead of re-planning.
    int dev = 0;
    cudaGetDevice(&dev);
    using Key = std::tuple<int, const uint8_t*, uint32_t, int, int, int, const float*, long long, float*, long long,
                           void*>;
    static std::mutex mu;
    static std::map<Key, eng::Plan> cache;
    const Key key{dev, w, type, n, d, B, x, ldx, out, ldo, ws};
    eng::Plan pl;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            pl = it->second;
        } else {
            eng::JobIn in{w, type, n, d, B, x, ldx, out, ldo};
            if (eng::make_plan(&in, 1, static_cast<uint8_t*>(ws), device_sm_count(), false, pl) != QUANTR_OK)
                return cudaErrorNotSupported;
            if (cache.size() >= 4096) cache.clear();
            cache.emplace(key, pl);
        }
    }
    return eng::launch_plan(pl, nullptr, err, stream);
}

size_t engine_act_bytes(uint32_t type, int d, int B) { return eng::act_bytes_for(type, d, B); }

} // namespace qr

// ----------------------------------------------------------- program API --

// Jobs with B >= kTcMinB tokens (up to kTcMaxB) run on the tensor-core kernel
// (tc.cu), the others on the dp4a engine above.
#ifndef QR_TC_MIN_B
#define QR_TC_MIN_B 2
#endif
constexpr int kTcMinB = QR_TC_MIN_B;

struct quantr_program {
    int device;
    bool has_engine = false;
    bool external_quant = false;  // the engine's inputs are quantized by the caller
    qr::eng::Plan plan;  // sub-plans own their device job tables
    qr::eng::QTask* d_tasks = nullptr;
    uint8_t* d_act = nullptr;
    std::vector<qr::TcPlan*> tc;  // tensor-core launches (<= kTcMaxJobs jobs each)
};

extern "C" {

int quantr_program_create(quantr_program** out, const quantr_gemv_job* jobs, int njobs)
{
    if (!out || !jobs || njobs <= 0) return QUANTR_ERR_BAD_ARG;
    std::vector<const float*> none((size_t)njobs, nullptr);
    return qr::program_create_ex(out, jobs, none.data(), njobs);
}

} // extern "C"

int qr::program_act_targets(const quantr_program* p, const float* x, ActTarget* out, int max)
{
    if (!p || !p->has_engine) return 0;
    int n = 0;
    for (const eng::QTask& t : p->plan.tasks)
        if (t.x == x && n < max) out[n++] = ActTarget{t.act, t.ds_off, t.U, t.B, t.type};
    return n;
}

int qr::program_external_quant(quantr_program* p, bool on)
{
    if (!p || !p->has_engine || !p->tc.empty()) return QUANTR_ERR_BAD_ARG;
    for (const eng::QTask& t : p->plan.tasks)
        if (t.xmul || t.B != 1) return QUANTR_ERR_BAD_ARG;
    p->external_quant = on;
    return QUANTR_OK;
}

int qr::program_create_ex(quantr_program** out, const quantr_gemv_job* jobs, const float* const* xmul, int njobs)
{
    using namespace qr;
    if (!out || !jobs || njobs <= 0) return QUANTR_ERR_BAD_ARG;
    *out = nullptr;
    std::vector<eng::JobIn> in;
    std::vector<GemvJobIn> tcj;
    for (int j = 0; j < njobs; ++j) {
        const quantr_gemv_job& J = jobs[j];
        const float* xm = xmul ? xmul[j] : nullptr;
        if (J.B > kTcMaxB && J.type != T_F32 && J.x && J.out && J.ldx >= J.d && J.ldo >= J.n) {
            // Wider jobs (a prefill chunk) run as kTcMaxB-token slices of the
            // same weights: tokens [b0, b0 + Bs) of x and out.
            for (int b0 = 0; b0 < J.B; b0 += kTcMaxB) {
                GemvJobIn g{static_cast<const uint8_t*>(J.w), J.type, J.n, J.d, std::min(kTcMaxB, J.B - b0),
                            J.x + (long long)b0 * J.ldx, J.ldx, J.out + (long long)b0 * J.ldo, J.ldo};
                g.xmul = xm ? xm + (long long)b0 * J.ldx : nullptr;
                tcj.push_back(g);
            }
        } else if (J.B >= kTcMinB && J.B <= kTcMaxB && J.type != T_F32) {
            GemvJobIn g{static_cast<const uint8_t*>(J.w), J.type, J.n, J.d, J.B, J.x, J.ldx, J.out, J.ldo};
            g.xmul = xm;
            tcj.push_back(g);
        } else {
            eng::JobIn e{static_cast<const uint8_t*>(J.w), J.type, J.n, J.d, J.B, J.x, J.ldx, J.out, J.ldo};
            e.xmul = xm;
            in.push_back(e);
        }
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return QUANTR_ERR_NO_DEVICE;
    }
    const int sms = device_sm_count();
    tc_split_narrow(tcj, sms);
    eng::Plan sizing;
    int rc = in.empty() ? QUANTR_OK : eng::make_plan(in.data(), (int)in.size(), nullptr, sms, true, sizing);
    if (rc) return rc;
    quantr_program* p = new (std::nothrow) quantr_program();
    if (!p) return QUANTR_ERR_OOM;
    p->device = dev;
    p->has_engine = !in.empty();
    for (size_t j0 = 0; j0 < tcj.size(); j0 += kTcMaxJobs) {
        TcPlan* tp = nullptr;
        rc = tc_plan_create(tcj.data() + j0, (int)std::min<size_t>(kTcMaxJobs, tcj.size() - j0), &tp);
        if (rc) {
            quantr_program_destroy(p);
            return rc;
        }
        p->tc.push_back(tp);
    }
    if (!p->has_engine) {
        *out = p;
        return QUANTR_OK;
    }
    if (cudaMalloc((void**)&p->d_act, std::max<size_t>(sizing.act_total, 256)) != cudaSuccess) {
        cudaGetLastError();
        p->d_act = nullptr;
        quantr_program_destroy(p);
        return QUANTR_ERR_OOM;
    }
    rc = eng::make_plan(in.data(), (int)in.size(), p->d_act, sms, true, p->plan);
    cudaError_t e = cudaSuccess;
    if (!rc) {
        e = cudaMalloc((void**)&p->d_tasks, p->plan.tasks.size() * sizeof(eng::QTask));
        if (e == cudaSuccess)
            e = cudaMemcpy(p->d_tasks, p->plan.tasks.data(), p->plan.tasks.size() * sizeof(eng::QTask),
                           cudaMemcpyHostToDevice);
        // Every sub-plan keeps a job table (even with one job), so a program
        // run never depends on host-side state.
        for (auto& sp : p->plan.subs) {
            if (e != cudaSuccess) break;
            e = cudaMalloc((void**)&sp.d_jobs, sp.jobs.size() * sizeof(eng::JobDesc));
            if (e == cudaSuccess)
                e = cudaMemcpy(sp.d_jobs, sp.jobs.data(), sp.jobs.size() * sizeof(eng::JobDesc),
                               cudaMemcpyHostToDevice);
        }
        if (e != cudaSuccess) rc = e == cudaErrorMemoryAllocation ? QUANTR_ERR_OOM : QUANTR_ERR_CUDA;
    }
    if (rc) {
        cudaGetLastError();
        quantr_program_destroy(p);
        return rc;
    }
    *out = p;
    return QUANTR_OK;
}

extern "C" {

int quantr_program_run(quantr_program* p, void* stream)
{
    if (!p) return QUANTR_ERR_BAD_ARG;
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != p->device) return QUANTR_ERR_BAD_ARG;
    int* err = qr::device_error_word();
    cudaError_t e = cudaSuccess;
    if (p->has_engine)
        e = qr::eng::launch_plan(p->plan, p->d_tasks, err, static_cast<cudaStream_t>(stream), p->external_quant);
    for (auto* tp : p->tc)
        if (e == cudaSuccess) e = qr::tc_plan_run(tp, err, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return QUANTR_ERR_CUDA;
    }
    return QUANTR_OK;
}

void quantr_program_destroy(quantr_program* p)
{
    if (!p) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaDeviceSynchronize();
    for (auto& sp : p->plan.subs) cudaFree(sp.d_jobs);
    cudaFree(p->d_tasks);
    cudaFree(p->d_act);
    for (auto* tp : p->tc) qr::tc_plan_destroy(tp);
    if (prev >= 0) cudaSetDevice(prev);
    delete p;
}

int quantr_program_info(const quantr_program* p, int* items, int* grid, int* smem_bytes)
{
    if (!p) return QUANTR_ERR_BAD_ARG;
    int it = 0, g = 0;
    size_t sm = 0;
    for (auto& sp : p->plan.subs) {
        it += sp.pp.total_items;
        g = std::max(g, sp.grid);
        sm = std::max(sm, sp.smem);
    }
    for (auto* tp : p->tc) {
        int ti = 0, tg = 0, ts = 0;
        qr::tc_plan_info(tp, &ti, &tg, &ts);
        it += ti;
        g = std::max(g, tg);
        sm = std::max(sm, (size_t)ts);
    }
    if (items) *items = it;
    if (grid) *grid = g;
    if (smem_bytes) *smem_bytes = (int)sm;
    return QUANTR_OK;
}

} // extern "C"
