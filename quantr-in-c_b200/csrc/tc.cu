// tc.cu -- batched-token quantized GEMV on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in TMEM), sm_100a.
//
// Every output of the reference (src/quant.c:242-437) is a left-to-right fp32
// sum over 32-element units of a term computed from the unit's int32 dot
// product isum = sum(w_q * x_q).  Here one tcgen05.mma per unit computes isum
// for a 128-row x N-token tile exactly (M=128, K=32, int8 x int8 -> int32,
// no accumulation across units), and epilogue warps read it from TMEM and
// apply the reference's term and running sum in unit order with explicitly
// rounded fp32 operations.  The integer products leave the CUDA cores, which
// keep only the exact-term arithmetic the reference's semantics require.
//
// A launch runs a list of GEMV jobs (B <= 64 tokens each, N = B rounded up
// to 16 columns) cut into 128-row tiles, dealt by a static longest-first
// schedule to one persistent CTA per SM.  A tile's K dimension streams in
// stages of 8 units (one K-quant super-block, or 8 Q8_0 blocks) through three
// shared-memory rings: SW slots of packed weights (fetched ahead, so that
// latency hides behind several stages), SO slots of MMA operands (unpacked
// weight tiles and activation tiles, free again when the stage's MMAs are
// done) and SE slots of epilogue data (weight scales and activation records,
// free again when the stage's epilogue is done):
//
//   weights (warp 0)     lane 0, per stage: one 2-D TMA copy of the tile's
//                        packed weights (128 rows x one stage of bytes) for
//                        jobs whose rows are 16-byte aligned (Q4_K, Q5_K);
//   activations (last    lane 0, per stage: two cp.async.bulk copies, the
//     warp)              stage's activation operand tiles and per-(unit,
//                        token) scale records (a warp of its own: one lane
//                        waiting on a barrier would stall the other's path);
//   MMA (warp 1)         per unit: tcgen05.mma (issued by one elected lane of
//                        the converged warp) into the stage's TMEM buffer (one
//                        of NBS, 8 units x N columns each); after the stage,
//                        one commit to the buffer's barrier and one that frees
//                        the operand slot;
//   decoders (4 warps)   for the other jobs, fetch the tile's packed bytes for
//                        the stage together (16-byte cp.async of each row's
//                        aligned segment cover, consecutive threads on
//                        consecutive chunks of a row, SW-1 stages ahead, one
//                        async-copy group per stage, a named barrier before
//                        use); then one thread per row
//                        unpacks each unit's quants into the canonical K-major
//                        no-swizzle operand layout (8x16-byte core matrices)
//                        and the unit's scales;
//   epilogue (4 x EG     TMEM lane quarter (warp % 4) x one of EG token
//     warps)             groups of NT tokens: per stage, tcgen05.ld of each
//                        unit's int32 sums for the group's live tokens (the
//                        next unit's load in flight while one is used), then
//                        term and running sum per (row, token), in unit
//                        order.  NT follows the launch's largest job (1, 2,
//                        4 or 8 tokens; 8 or 16 for wider jobs).
//
// Activations are quantized by k_tc_quant (quantize_row_q8_0 per token, the
// same kernel math as every other path) straight into operand tiles in the
// element order each weight type's decode produces, or arrive as operand
// tiles (gathered jobs: the pairs routed to one MoE expert, whose count and
// pair list an earlier launch writes; every role reads the count, skips
// experts nobody chose and runs one pass over the tile per 16 pairs).  Each
// launch runs a kernel built for its split, for whether it has gathered jobs,
// and for its weight type when all jobs share one (smaller code: instruction
// fetch was a leading stall of the generic kernel).  All waits are bounded
// (250 ms); on a timeout every role stops, copies in flight are drained, the
// last MMAs are awaited and TMEM is freed before the CTA exits.  No multicast.
#include "quantr_cuda.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include "device_common.cuh"
#include "formats.cuh"
#include "kernels.cuh"
#include "launch_util.cuh"
#include "libm_ref.cuh"
#include "quant_decode.cuh"

#include <algorithm>
#include <functional>
#include <map>
#include <new>
#include <queue>
#include <tuple>
#include <utility>
#include <vector>
#include <mutex>

namespace qr {
namespace tc {

constexpr int kM = 128;        // rows per tile (MMA M)
constexpr int kUS = 8;         // units per stage
constexpr int kGroupWarps = 4;  // one decoder thread per tile row in each decoder group
// Longest suspension (ns) of one barrier poll, per role: a waiting warp
// sleeps until its phase completes instead of spinning on issue slots.
#ifndef QR_TC_SUSPEND_EPI
#define QR_TC_SUSPEND_EPI 2000
#endif
#ifndef QR_TC_SUSPEND_MMA
#define QR_TC_SUSPEND_MMA 1000
#endif
#ifndef QR_TC_SUSPEND_PROD
#define QR_TC_SUSPEND_PROD 4000
#endif
#ifndef QR_TC_SUSPEND_DEC
#define QR_TC_SUSPEND_DEC 1000
#endif
#ifndef QR_TC_N16_EG
#define QR_TC_N16_EG 2
#endif
#ifndef QR_TC_B8_EG
#define QR_TC_B8_EG 2
#endif
#ifndef QR_TC_B4_EG
#define QR_TC_B4_EG 1
#endif
#ifndef QR_TC_N16_DG
#define QR_TC_N16_DG 2
#endif
constexpr unsigned kSleepEpi = QR_TC_SUSPEND_EPI, kSleepMma = QR_TC_SUSPEND_MMA, kSleepProd = QR_TC_SUSPEND_PROD,
                   kSleepDec = QR_TC_SUSPEND_DEC;
// Warp split of a launch: DG decoder groups of four warps taking alternate
// stages, and 4 TMEM lane quarters x EG epilogue token groups (NT tokens
// each) after the producer and MMA warps.  Launches whose jobs have at most 8
// tokens run <2, 1> with NT = the token count rounded up to a power of two
// (the MMA still computes N = 16 columns; the epilogue reads and evaluates
// only the live ones), up to 16 tokens <2, 2> with NT = 8, wider ones <1, 4>
// (epilogue-bound).
template <int DG, int EG>
struct Split {
    static constexpr int dec_warps = DG * kGroupWarps, epi_warps = 4 * EG;
    // + weight producer, MMA warp and (last) activation producer.  The two
    // producers are separate warps: lanes of one diverged warp that wait on
    // different barriers would hold each other up.
    static constexpr int threads = 32 * (3 + dec_warps + epi_warps);
};
constexpr int kMaxSW = 8;      // packed-weight slots
constexpr int kMaxSO = 2;      // unpacked weight tile slots (MMA A operands)
constexpr int kMaxSB = 8;      // activation tile slots (MMA B operands)
constexpr int kMaxSE = 4;      // epilogue slots (activation records and weight scales)
constexpr int kMaxNB = 4;      // TMEM stage buffers
constexpr int kMaxN = kTcMaxB; // tokens per job (MMA N after padding)
constexpr size_t kSmemMax = 227 * 1024;
constexpr uint32_t kATile = 4096;  // one unit's 128 x 32-byte operand tile

// One GEMV of a launch (device view).
struct __align__(16) TcJob {
    const uint8_t* w;      // packed rows (16-byte aligned base)
    const uint8_t* act;    // [U] x (N x 32-byte canonical operand tile)
    const uint8_t* ds;     // per unit: dx[N] | (float)bsum[N] | 32*bsum[N] (int) | unused[N]
    float* out;
    long long ldo;
    long long rb;          // packed row bytes
    uint32_t type, n, U, B;
    uint32_t N, nst, seg, idesc;  // nst stages of kUS units; seg = packed bytes of a full stage per row
    int tiles, item0;
    int tma;  // weights fetched by one 2-D TMA copy per stage (rows 16-byte aligned: Q4_K, Q5_K)
    int ge;   // gathered job (GemvJobIn): expert index into the launch's pair counts/lists; -1: dense
};
static_assert(sizeof(TcJob) % 16 == 0, "job table is copied in 16-byte words");
static_assert(sizeof(TcJob) == 96, "the job table lives in shared memory: keep it small");

struct TcParams {
    const TcJob* jobs;
    int njobs, total_items;
    uint32_t SW, SO, SB, SE, NB;           // weight, A-tile, B-tile and epilogue slots, TMEM stage buffers
    uint32_t ncol, tmem_cols;              // max N, TMEM columns
    uint32_t segp;                         // staging bytes per row of a weight slot (cp.async jobs)
    uint32_t w_off, w_slot;                // weight ring: first slot, bytes per slot
    uint32_t o_off, o_slot;                // A-tile ring: first slot, bytes per slot
    uint32_t b_off, b_slot;                // B-tile ring: first slot, bytes per slot
    uint32_t e_off, e_slot;                // epilogue ring: first slot, bytes per slot
    uint32_t d_rel, s_rel;                 // activation records, weight scales within an epilogue slot
    uint32_t jobs_off;
    // Static schedule: CTA c walks entries [sched_off[c], sched_off[c + 1]) of
    // sched, each (job << 20) | item, copied to shared memory at sched_smem.
    const uint32_t* sched;
    const int* sched_off;
    uint32_t sched_smem;
    int gathered;  // some job's live columns come from an earlier launch: every role waits for it
    // Gathered jobs' pair counts, list offsets and pair lists (one set per launch).
    const int* gcounts;
    const int* goffsets;
    const int* glist;
    int* err;
    // Per job with tma set: rows x row-bytes uint8 view of the packed weights,
    // box = 128 rows x one stage's bytes (passed by value: TMA reads the map
    // from the kernel's parameter space).
    CUtensorMap tmap[kTcMaxJobs];
};

// ------------------------------------------------------------ tcgen05 --

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr)
{
    // Canonical K-major, no swizzle: core matrices of 8 rows x 16 bytes; the
    // two K halves 128 bytes apart (LBO), 8-row groups 256 bytes apart (SBO);
    // descriptor version 1 (sm_100) at bit 46.
    uint64_t d = (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(128u >> 4) << 16;
    d |= (uint64_t)(256u >> 4) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc)
{
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sptr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t addr, uint32_t (&v)[NC]);

template <>
__device__ __forceinline__ void tmem_ld<1>(uint32_t addr, uint32_t (&v)[1])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n" : "=r"(v[0]) : "r"(addr));
}

template <>
__device__ __forceinline__ void tmem_ld<2>(uint32_t addr, uint32_t (&v)[2])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];\n" : "=r"(v[0]), "=r"(v[1]) : "r"(addr));
}

template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t addr, uint32_t (&v)[4])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(addr));
}

template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t addr, uint32_t (&v)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(addr));
}

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t addr, uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(addr));
}

template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t addr, uint32_t (&v)[32])
{
    uint32_t (&a)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[0]);
    uint32_t (&b)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[16]);
    tmem_ld<16>(addr, a);
    tmem_ld<16>(addr + 16, b);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// True in exactly one lane of the (converged) warp.
__device__ __forceinline__ bool elect_one()
{
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(pred));
    return pred != 0;
}

// ------------------------------------------------------------- quantizer --

struct TcQTask {
    const float* x;
    const float* xmul;  // non-null: the input is silu(x) * xmul, elementwise
    uint8_t* act;
    uint8_t* ds;
    long long ldx;
    long long blk0;  // first global (unit, token) index of this task
    int U, B, N, type;
    int vec;  // x rows start 16-byte aligned: 128-bit loads
    int pad;
};

struct TcQParams {
    const TcQTask* tasks;
    int ntasks;
    long long total;
};

// Position of element e (0..31) of a unit in the element order the weight
// type's decode produces (quant_decode.cuh permute_x16).
__device__ __forceinline__ int tc_perm(int type, int e)
{
    if (type == T_Q4_K || type == T_Q5_K) return (e & ~7) + ((e & 1) << 2) + ((e & 7) >> 1);
    if (type == T_Q6_K) return (e & ~15) + ((e & 3) << 2) + ((e & 15) >> 2);
    return e;
}

// quantize_row_q8_0's rounding of one scaled value to the int8 it stores:
// x86 lrintf (round to nearest even) truncated to 8 bits, where NaN and
// out-of-range inputs give 0x8000000000000000 (low byte 0).  For |v| >= 2^31
// every float is a multiple of 2^8, whose low byte is 0 as well.
__device__ __forceinline__ uint32_t q8_round_byte(float v)
{
    return fabsf(v) < 2147483648.0f ? ((uint32_t)__float2int_rn(v) & 0xFFu) : 0u;
}

// Reference quantize_row_q8_0 (src/quant.c:143) per (token, 32-element
// block), one thread per block, written into canonical operand tiles: token
// t, permuted element k of unit u at u*N*32 + (t/8)*256 + (t%8)*16 +
// (k/16)*128 + k%16.  Threads take blocks token-fastest within a unit, so a
// warp's tile stores and record stores are contiguous.
__global__ void __launch_bounds__(256) k_tc_quant(const __grid_constant__ TcQParams p)
{
    // The task table (written once, at plan time) goes to shared memory before
    // the wait for the previous grid, so the per-block task search below reads
    // no global memory.
    static_assert(sizeof(TcQTask) % 8 == 0, "task table is copied in 8-byte words");
    __shared__ TcQTask tasks[kTcMaxJobs];
    pdl_trigger();
    {
        const long long* src = reinterpret_cast<const long long*>(p.tasks);
        long long* dst = reinterpret_cast<long long*>(tasks);
        const int words = p.ntasks * (int)(sizeof(TcQTask) / 8);
        for (int w = threadIdx.x; w < words; w += blockDim.x) dst[w] = src[w];
    }
    __syncthreads();
    pdl_wait();
    const long long step = (long long)gridDim.x * blockDim.x;
    for (long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < p.total; g += step) {
        int ti = 0, hi = p.ntasks - 1;  // last task with blk0 <= g
        while (ti < hi) {
            const int mid = (ti + hi + 1) >> 1;
            if (tasks[mid].blk0 <= g) ti = mid; else hi = mid - 1;
        }
        const TcQTask& T = tasks[ti];
        const int local = (int)(g - T.blk0);  // < B * U
        const int u = local / T.B, t = local - u * T.B;
        const float* src = T.x + (long long)t * T.ldx + (long long)u * 32;
        float v[32];
        if (T.vec) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 f = reinterpret_cast<const float4*>(src)[i];
                v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = src[i];
        }
        if (T.xmul) {
            const float* m3 = T.xmul + (long long)t * T.ldx + (long long)u * 32;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = libm::swiglu_ref(v[i], m3[i]);
        }
        // amax = max |x| over the block, NaN ignored (src/quant.c:149-152).
        uint32_t abits = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float a = fabsf(v[i]);
            abits = max(abits, (a == a) ? __float_as_uint(a) : 0u);
        }
        const float dd = __fdiv_rn(__uint_as_float(abits), 127.0f);
        const float id = (dd != 0.0f) ? __fdiv_rn(1.0f, dd) : 0.0f;
        uint32_t q[32];
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            q[i] = q8_round_byte(__fmul_rn(v[i], id));
            sum += (int)(int8_t)q[i];
        }
        // Element e goes to byte tc_perm(type, e) of the unit's 32 bytes.
        uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (T.type == T_Q4_K || T.type == T_Q5_K) {
#pragma unroll
            for (int e = 0; e < 32; ++e) w[tc_perm(T_Q4_K, e) >> 2] |= q[e] << (8 * (tc_perm(T_Q4_K, e) & 3));
        } else if (T.type == T_Q6_K) {
#pragma unroll
            for (int e = 0; e < 32; ++e) w[tc_perm(T_Q6_K, e) >> 2] |= q[e] << (8 * (tc_perm(T_Q6_K, e) & 3));
        } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) w[e >> 2] |= q[e] << (8 * (e & 3));
        }
        uint8_t* tile = T.act + (size_t)u * T.N * 32 + (t >> 3) * 256 + (t & 7) * 16;
        *reinterpret_cast<uint4*>(tile) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(tile + 128) = make_uint4(w[4], w[5], w[6], w[7]);
        float* rec = reinterpret_cast<float*>(T.ds) + (size_t)u * T.N * 4;  // planar per unit: dx | bsum | 32*bsum
        rec[t] = h2f_ref(f2h_ref(dd));
        rec[T.N + t] = (float)sum;
        rec[2 * T.N + t] = __int_as_float(32 * sum);
    }
}

// Passes of an item over its K stages: 1 for a dense job; for a gathered job
// (the pairs routed to one MoE expert, count written by an earlier launch and
// read after the dependency wait) one per N live columns, 0 when it has none.
// Every role derives the same value, so all of them walk the same stages.
// GAT: the launch has gathered jobs (a separate kernel instantiation, so that
// dense launches keep single-pass loops).
template <bool GAT>
__device__ __forceinline__ int job_passes(const TcParams& p, const TcJob& J)
{
    if constexpr (!GAT) return 1;
    return J.ge >= 0 ? (p.gcounts[J.ge] + (int)J.N - 1) / (int)J.N : 1;
}
// Live columns of pass `pass`.
template <bool GAT>
__device__ __forceinline__ int pass_live(const TcParams& p, const TcJob& J, int pass)
{
    if constexpr (!GAT) return (int)J.B;
    return J.ge >= 0 ? min((int)J.N, p.gcounts[J.ge] - pass * (int)J.N) : (int)J.B;
}

// This CTA's schedule: entry k = (job << 20) | item.
struct Sched {
    const uint32_t* list;
    int cnt;
    __device__ __forceinline__ int item(int k) const { return (int)(list[k] & 0xFFFFFu); }
    __device__ __forceinline__ int job(int k) const { return (int)(list[k] >> 20); }
};

// Term and running sum of one unit for this warp's NT tokens (v = the unit's
// int32 sums from TMEM; scale_at = this row's (scale, min) pair, rec_at = the
// unit's activation scales for the warp's first token, aux_off = the distance
// to its bsum or 32*bsum records).  Padding tokens (>= B) have zero
// activations and records, so they are computed without branches and never
// stored.  Shared memory is read through 32-bit shared-window addresses.
template <uint32_t TYPE, int NT>
__device__ __forceinline__ void epi_unit(const uint32_t (&v)[NT], uint32_t scale_at, uint32_t rec_at,
                                         uint32_t aux_off, float (&acc)[NT])
{
    const uint2 scm = lds64(scale_at);
    const float sc = __uint_as_float(scm.x), m = __uint_as_float(scm.y);
    if constexpr (NT < 4) {  // one or two tokens: word loads of the records
#pragma unroll
        for (int q = 0; q < NT; ++q) {
            const int isum = (int)v[q];
            const float d = __uint_as_float(lds32(rec_at + (uint32_t)q * 4));
            const uint32_t ax = TYPE != T_Q8_0 ? lds32(rec_at + aux_off + (uint32_t)q * 4) : 0u;
            float term;
            if (TYPE == T_Q8_0) term = __fmul_rn(__fmul_rn((float)isum, sc), d);  // src/quant.c:284
            else if (TYPE == T_Q6_K) term = __fmul_rn(__fmul_rn(sc, (float)(isum - (int)ax)), d);  // :433
            else term = __fmul_rn(__fsub_rn(__fmul_rn(sc, (float)isum), __fmul_rn(m, __uint_as_float(ax))), d);  // :399
            acc[q] = __fadd_rn(acc[q], term);
        }
        return;
    }
#pragma unroll
    for (int t4 = 0; t4 < NT; t4 += 4) {
        const uint4 dx = lds128(rec_at + (uint32_t)t4 * 4);
        uint4 aux = make_uint4(0, 0, 0, 0);
        if (TYPE != T_Q8_0) aux = lds128(rec_at + aux_off + (uint32_t)t4 * 4);  // bsum | 32*bsum
        const uint32_t dxa[4] = {dx.x, dx.y, dx.z, dx.w}, ax[4] = {aux.x, aux.y, aux.z, aux.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int isum = (int)v[t4 + q];
            const float d = __uint_as_float(dxa[q]);
            float term;
            if (TYPE == T_Q8_0) term = __fmul_rn(__fmul_rn((float)isum, sc), d);  // src/quant.c:284
            else if (TYPE == T_Q6_K) term = __fmul_rn(__fmul_rn(sc, (float)(isum - (int)ax[q])), d);  // :433
            else term = __fmul_rn(__fsub_rn(__fmul_rn(sc, (float)isum), __fmul_rn(m, __uint_as_float(ax[q]))), d);  // :399
            acc[t4 + q] = __fadd_rn(acc[t4 + q], term);
        }
    }
}

// One stage of the epilogue over us units (FULL: all kUS, straight-line code
// with compile-time offsets).  The TMEM load of unit j+1 is in flight while
// unit j's terms are computed (two register buffers; one for NT >= 16).
// scale0 / rec0: unit 0's scale pair of this row and records of this warp's
// first token.
template <uint32_t TYPE, int NT, bool FULL>
__device__ __forceinline__ void epi_stage(uint32_t tbase, uint32_t scale0, uint32_t rec0, int N, int us,
                                          float (&acc)[NT])
{
    const uint32_t aux_off = (TYPE == T_Q6_K ? 8u : 4u) * (uint32_t)N;  // records: dx[N] | bsum[N] | 32*bsum[N]
    const uint32_t rec_step = 16u * (uint32_t)N;
    constexpr uint32_t sc_step = kM * 8;
    if constexpr (FULL) {
        if constexpr (NT >= 16) {
#pragma unroll
            for (int j = 0; j < kUS; ++j) {
                uint32_t v[NT];
                tmem_ld<NT>(tbase + (uint32_t)(j * N), v);
                tmem_wait_ld();
                epi_unit<TYPE, NT>(v, scale0 + j * sc_step, rec0 + j * rec_step, aux_off, acc);
            }
        } else {
            uint32_t v[2][NT];
            tmem_ld<NT>(tbase, v[0]);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < kUS; ++j) {
                if (j + 1 < kUS) tmem_ld<NT>(tbase + (uint32_t)((j + 1) * N), v[(j + 1) & 1]);
                epi_unit<TYPE, NT>(v[j & 1], scale0 + j * sc_step, rec0 + j * rec_step, aux_off, acc);
                if (j + 1 < kUS) tmem_wait_ld();
            }
        }
    } else {
        for (int j = 0; j < us; ++j) {
            uint32_t v[NT];
            tmem_ld<NT>(tbase + (uint32_t)(j * N), v);
            tmem_wait_ld();
            epi_unit<TYPE, NT>(v, scale0 + j * sc_step, rec0 + j * rec_step, aux_off, acc);
        }
    }
}

struct Bars {
    uint64_t *wfull, *wempty;         // weight ring: filled (TMA or decoders' own copies), free again
    uint64_t *afull, *ofree;          // A-tile ring: tiles written, MMAs done
    uint64_t *bfull, *bfree;          // B-tile ring: tiles landed, MMAs done
    uint64_t *dfull, *sfull, *efree;  // epilogue ring: records landed, scales written, epilogue done
    uint64_t *t_full, *t_empty;       // TMEM stage buffers: sums ready, read
};

template <int NT, int DW, bool GAT, int TY>
__device__ void epilogue_role(uint8_t* sm, const TcParams& p, const TcJob* jobs, const Sched& sc, const Bars& br,
                              volatile int* abort_flag, uint32_t tmem, int warp, int lane)
{
    const int quarter = warp & 3, grp = (warp - 2 - DW) >> 2;
    const int row = 32 * quarter + lane;
    const int SE = (int)p.SE, NB = (int)p.NB;
    const int tok0 = grp * NT;
    const uint32_t tq = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)tok0;  // this warp's lanes and tokens
    const uint32_t e0 = sptr(sm) + p.e_off, srow = p.s_rel + (uint32_t)row * 8, drow = p.d_rel + (uint32_t)tok0 * 4;
    // Stage gs's epilogue slot es (used eu times before) and TMEM buffer sb
    // (used bu times before).
    int es = 0, eu = 0, sb = 0, bu = 0;
    bool ok = true;
    for (int k = 0; ok && k < sc.cnt; ++k) {
        const int i = sc.item(k);
        const TcJob& J = jobs[sc.job(k)];
        const int r0 = (i - J.item0) * kM;
        const int rows = min(kM, (int)J.n - r0);
        const int N = (int)J.N, U = (int)J.U, nst = (int)J.nst;
        const uint32_t type = J.type;
        float* out = J.out;
        const long long ldo = J.ldo;
        const int npass = job_passes<GAT>(p, J);
        for (int pass = 0; ok && pass < npass; ++pass) {
            const int B = pass_live<GAT>(p, J, pass);  // live columns of this pass
            float acc[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
            for (int st = 0; st < nst; ++st) {
                if (!mbar_wait_bounded(&br.dfull[es], eu & 1, p.err, abort_flag, kSleepEpi) ||
                    !mbar_wait_bounded(&br.sfull[es], eu & 1, p.err, abort_flag, kSleepEpi) ||
                    !mbar_wait_bounded(&br.t_full[sb], bu & 1, p.err, abort_flag, kSleepEpi)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ebase = e0 + p.e_slot * (uint32_t)es;
                const int us = min(kUS, U - kUS * st);
                const uint32_t tbase = tq + (uint32_t)(sb * kUS) * p.ncol;
                if (tok0 < B) {
                    const uint32_t s0 = ebase + srow, r0b = ebase + drow;
                    if constexpr (TY == T_Q4_K || TY == T_Q5_K || TY == T_Q6_K) {
                        // One K-quant type: a row is whole super-blocks, every stage is full.
                        epi_stage<(uint32_t)TY, NT, true>(tbase, s0, r0b, N, us, acc);
                    } else if constexpr (TY >= 0) {  // one weight type in the launch: its code only
                        if (us == kUS) epi_stage<(uint32_t)TY, NT, true>(tbase, s0, r0b, N, us, acc);
                        else epi_stage<(uint32_t)TY, NT, false>(tbase, s0, r0b, N, us, acc);
                    } else if (us == kUS) {
                        switch (type) {
                        case T_Q4_K: epi_stage<T_Q4_K, NT, true>(tbase, s0, r0b, N, us, acc); break;
                        case T_Q5_K: epi_stage<T_Q5_K, NT, true>(tbase, s0, r0b, N, us, acc); break;
                        case T_Q6_K: epi_stage<T_Q6_K, NT, true>(tbase, s0, r0b, N, us, acc); break;
                        default: epi_stage<T_Q8_0, NT, true>(tbase, s0, r0b, N, us, acc); break;
                        }
                    } else {
                        switch (type) {
                        case T_Q4_K: epi_stage<T_Q4_K, NT, false>(tbase, s0, r0b, N, us, acc); break;
                        case T_Q5_K: epi_stage<T_Q5_K, NT, false>(tbase, s0, r0b, N, us, acc); break;
                        case T_Q6_K: epi_stage<T_Q6_K, NT, false>(tbase, s0, r0b, N, us, acc); break;
                        default: epi_stage<T_Q8_0, NT, false>(tbase, s0, r0b, N, us, acc); break;
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&br.t_empty[sb]);
                    mbar_arrive(&br.efree[es]);
                }
                if (++es == SE) es = 0, ++eu;
                if (++sb == NB) sb = 0, ++bu;
            }
            if (!ok) break;
            if (row < rows) {
                // Output row of column t: the token (dense job) or the pair
                // the gathered column stands for.
                const int* lst = GAT && J.ge >= 0 ? p.glist + p.goffsets[J.ge] + pass * N : nullptr;
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    if (tok0 + t < B)
                        out[(long long)(lst ? lst[tok0 + t] : tok0 + t) * ldo + r0 + row] = acc[t];
            }
        }
    }
}

// A 16-byte aligned Q4_K/Q5_K super-block (shared-memory offset sb) into the
// stage's 8 operand tiles (row offset arow) and scales (srow): the element
// order of quant_decode.cuh decode_unit, read with 128-bit loads.
template <uint32_t TYPE>
__device__ __forceinline__ void decode_k45_aligned(uint8_t* sm, uint32_t sb, uint32_t arow, uint32_t srow)
{
    const uint4 hdr = *reinterpret_cast<const uint4*>(sm + sb);
    const float d = h2f_ref(hdr.x & 0xFFFFu), dmin = h2f_ref(hdr.x >> 16);
    uint4 qh0 = make_uint4(0, 0, 0, 0), qh1 = qh0;
    if (TYPE == T_Q5_K) {
        qh0 = *reinterpret_cast<const uint4*>(sm + sb + 16);
        qh1 = *reinterpret_cast<const uint4*>(sm + sb + 32);
    }
    const uint32_t qs = sb + (TYPE == T_Q4_K ? 16u : 48u);
    // Every load before the first store: the stores go through the same
    // shared-memory pointer, so the compiler would otherwise keep each
    // unit's load behind the previous unit's stores.
    uint4 q8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) q8[j] = *reinterpret_cast<const uint4*>(sm + qs + 16 * j);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t scb = ((j < 4 ? hdr.y : hdr.z) >> (8 * (j & 3))) & 0xFFu;
        const float sc = __fmul_rn((float)(scb & 63u), d);   // src/quant.c:385
        const float m = __fmul_rn((float)(scb >> 6), dmin);  // src/quant.c:386
        const uint32_t qw[4] = {q8[j].x, q8[j].y, q8[j].z, q8[j].w};
        uint32_t wq[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wq[2 * i] = qw[i] & 0x0F0F0F0Fu;
            wq[2 * i + 1] = (qw[i] >> 4) & 0x0F0F0F0Fu;
        }
        if (TYPE == T_Q5_K) {
            const uint32_t H = (j < 4) ? (j == 0 ? qh0.x : j == 1 ? qh0.y : j == 2 ? qh0.z : qh0.w)
                                       : (j == 4 ? qh1.x : j == 5 ? qh1.y : j == 6 ? qh1.z : qh1.w);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t hb = (H >> (8 * i)) & 0xFFu;
                wq[2 * i] |= spread_even_bits_to_b4(hb);
                wq[2 * i + 1] |= spread_even_bits_to_b4(hb >> 1);
            }
        }
        uint4* at = reinterpret_cast<uint4*>(sm + arow + (uint32_t)j * kATile);
        at[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
        at[8] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
        *reinterpret_cast<float2*>(sm + srow + (uint32_t)j * kM * 8) = make_float2(sc, m);
    }
}

// The us (<= 8) units of a row segment at seg0 with the generic per-unit
// decoder (Q6_K, Q8_0 and rows that are not 16-byte aligned).
template <uint32_t TYPE>
__device__ __forceinline__ void decode_units(const uint32_t* s32, uint8_t* sm, uint32_t seg0, int us, uint32_t arow,
                                             uint32_t srow)
{
    for (int j = 0; j < us; ++j) {
        Unit o;
        decode_unit<TYPE>(s32, sm, seg0, j, o);
        uint4* at = reinterpret_cast<uint4*>(sm + arow + (uint32_t)j * kATile);
        at[0] = make_uint4(o.wq[0], o.wq[1], o.wq[2], o.wq[3]);
        at[8] = make_uint4(o.wq[4], o.wq[5], o.wq[6], o.wq[7]);
        *reinterpret_cast<float2*>(sm + srow + (uint32_t)j * kM * 8) = make_float2(o.a, o.b);
    }
}

// cp.async.wait_group with the immediate n = SW - 2 (all but the newest
// SW - 2 groups complete).
__device__ __forceinline__ void wait_groups_but(int n)
{
    switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    }
}

// TY: the weight type of every job in the launch (its decode and epilogue
// code only), or -1 for launches that mix types.
template <int DG, int EG, int NT, bool GAT, int TY>
__global__ void __launch_bounds__(Split<DG, EG>::threads, 1) k_tc_program(const __grid_constant__ TcParams p)
{
    constexpr int kDecWarps = Split<DG, EG>::dec_warps, kEpiWarps = Split<DG, EG>::epi_warps;
    constexpr int kThreads = Split<DG, EG>::threads;
    extern __shared__ __align__(1024) uint8_t sm[];
    Bars br;
    br.wfull = reinterpret_cast<uint64_t*>(sm);
    br.wempty = br.wfull + kMaxSW;
    br.afull = br.wempty + kMaxSW;
    br.ofree = br.afull + kMaxSO;
    br.bfull = br.ofree + kMaxSO;
    br.bfree = br.bfull + kMaxSB;
    br.dfull = br.bfree + kMaxSB;
    br.sfull = br.dfull + kMaxSE;
    br.efree = br.sfull + kMaxSE;
    br.t_full = br.efree + kMaxSE;
    br.t_empty = br.t_full + kMaxNB;
    // [0] TMEM base, [1] abort, then the bulk/TMA fills issued so far per
    // weight slot [kFillW..), B-tile slot [kFillB..) and record slot [kFillD..).
    constexpr int kFillW = 2, kFillB = kFillW + kMaxSW, kFillD = kFillB + kMaxSB;
    uint32_t* misc = reinterpret_cast<uint32_t*>(br.t_empty + kMaxNB);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int SW = (int)p.SW, SO = (int)p.SO, SB = (int)p.SB, SE = (int)p.SE, NB = (int)p.NB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SW; ++s) {
            mbar_init(&br.wfull[s], 1);
            mbar_init(&br.wempty[s], kGroupWarps);
            misc[kFillW + s] = 0;
        }
        for (int s = 0; s < SO; ++s) {
            mbar_init(&br.afull[s], kGroupWarps);
            mbar_init(&br.ofree[s], 1);
        }
        for (int s = 0; s < SB; ++s) {
            mbar_init(&br.bfull[s], 1);
            mbar_init(&br.bfree[s], 1);
            misc[kFillB + s] = 0;
        }
        for (int s = 0; s < SE; ++s) {
            mbar_init(&br.dfull[s], 1);
            mbar_init(&br.sfull[s], kGroupWarps);
            mbar_init(&br.efree[s], kEpiWarps);
            misc[kFillD + s] = 0;
        }
        for (int b = 0; b < NB; ++b) {
            mbar_init(&br.t_full[b], 1);
            mbar_init(&br.t_empty[b], kEpiWarps);
        }
        misc[1] = 0;
        mbar_fence_init();
    }
    {  // job table -> shared memory
        const uint4* src = reinterpret_cast<const uint4*>(p.jobs);
        uint4* dst = reinterpret_cast<uint4*>(sm + p.jobs_off);
        const int words = p.njobs * (int)(sizeof(TcJob) / 16);
        for (int w = threadIdx.x; w < words; w += kThreads) dst[w] = src[w];
    }
    Sched sc;
    {  // this CTA's schedule -> shared memory
        const int s0 = p.sched_off[blockIdx.x];
        sc.cnt = p.sched_off[blockIdx.x + 1] - s0;
        uint32_t* dst = reinterpret_cast<uint32_t*>(sm + p.sched_smem);
        for (int w = threadIdx.x; w < sc.cnt; w += kThreads) dst[w] = p.sched[s0 + w];
        sc.list = dst;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sptr(&misc[0])),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];
    const TcJob* jobs = reinterpret_cast<const TcJob*>(sm + p.jobs_off);
    pdl_trigger();
    // Gathered jobs' live-column counts come from an earlier launch: every role
    // needs them to skip the same items.
    if (GAT) pdl_wait();

    if (warp == 0) {
        // ----------------------------------------------- weight producer --
        if (lane == 0) {
            // Weight ring: waits for every stage's slot (so it never runs more
            // than SW stages ahead of the decoders), copies the TMA jobs'.
            // Weights do not depend on the previous grid: no PDL wait.
            int ws = 0, wu = 0;  // this stage's weight slot, earlier uses of it
            bool ok = true;
            for (int k = 0; ok && k < sc.cnt; ++k) {
                const int i = sc.item(k), jc = sc.job(k);
                const TcJob& J = jobs[jc];
                const int nps = job_passes<GAT>(p, J) * (int)J.nst;  // (pass, stage) steps; each pass re-reads the tile
                // Counters, not divisions: this single thread is on every stage's critical path.
                for (int ps = 0, st = 0; ps < nps;
                     ++ps, (++st == (int)J.nst ? st = 0 : 0), (++ws == SW ? (ws = 0, ++wu) : 0)) {
                    if (wu > 0 && !mbar_wait_bounded(&br.wempty[ws], (wu - 1) & 1, p.err, abort_flag, kSleepProd)) {
                        ok = false;
                        break;
                    }
                    misc[kFillW + ws] += 1;  // one arrival per use keeps the slot's phases = its uses
                    if (!J.tma) {
                        mbar_arrive(&br.wfull[ws]);  // the decoders fetch this stage themselves
                    } else {  // box (x = byte offset in the row, a multiple of 16; y = first row)
                        mbar_arrive_expect_tx(&br.wfull[ws], J.seg * (uint32_t)kM);
                        const int x = st * (int)J.seg, y = (i - J.item0) * kM;
                        asm volatile(
                            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
                            "[%0], [%1, {%2, %3}], [%4];" ::"r"(sptr(sm + p.w_off + p.w_slot * (uint32_t)ws)),
                            "l"(reinterpret_cast<uint64_t>(&p.tmap[jc])), "r"(x), "r"(y), "r"(sptr(&br.wfull[ws]))
                            : "memory");
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA --
        // The whole warp walks the stages (converged); one elected lane issues.
        int last_sb = -1, last_ph = 0;
        // This stage's A slot, B slot and TMEM buffer, and earlier uses of them.
        int os = 0, ou = 0, bs = 0, bsu = 0, sb = 0, bu = 0;
        bool ok = true;
        for (int k = 0; ok && k < sc.cnt; ++k) {
            const TcJob& J = jobs[sc.job(k)];
            const int nps = job_passes<GAT>(p, J) * (int)J.nst;
            for (int ps = 0, st = 0; ps < nps; ++ps, (++st == (int)J.nst ? st = 0 : 0), (++os == SO ? (os = 0, ++ou) : 0),
                     (++bs == SB ? (bs = 0, ++bsu) : 0), (++sb == NB ? (sb = 0, ++bu) : 0)) {
                if (!mbar_wait_bounded(&br.bfull[bs], bsu & 1, p.err, abort_flag, kSleepMma) ||
                    !mbar_wait_bounded(&br.afull[os], ou & 1, p.err, abort_flag, kSleepMma) ||
                    (bu > 0 && !mbar_wait_bounded(&br.t_empty[sb], (bu - 1) & 1, p.err, abort_flag, kSleepMma))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                __syncwarp();
                const uint32_t abase = p.o_off + p.o_slot * (uint32_t)os, bbase = p.b_off + p.b_slot * (uint32_t)bs;
                const int us = min(kUS, (int)J.U - kUS * st);
                if (elect_one()) {
                    for (int j = 0; j < us; ++j) {
                        const uint64_t ad = smem_desc(sptr(sm + abase + (uint32_t)j * kATile));
                        const uint64_t bd = smem_desc(sptr(sm + bbase + (uint32_t)(j * (int)J.N) * 32u));
                        tc_mma(tmem + (uint32_t)(sb * kUS * (int)p.ncol + j * (int)J.N), ad, bd, J.idesc);
                    }
                    tc_commit(&br.t_full[sb]);
                    tc_commit(&br.ofree[os]);
                    tc_commit(&br.bfree[bs]);
                }
                __syncwarp();
                last_sb = sb;
                last_ph = bu & 1;
            }
        }
        // The MMAs issued last complete before TMEM is released.
        if (last_sb >= 0) mbar_wait_bounded(&br.t_full[last_sb], (uint32_t)last_ph, nullptr);
        __syncwarp();
    } else if (warp < 2 + kDecWarps) {
        // ------------------------------------------------------ decoders --
        // DG groups of four warps take alternate stages (group grp the stages
        // gs with gs % DG == grp): one group's waits and decode overlap the
        // other's.  One thread per tile row within a group.
        static_assert(DG == 1 || (DG == 2 && kMaxSO == 2), "with two groups each keeps one A slot");
        const int grp = (warp - 2) / kGroupWarps;
        const int row = ((warp - 2) % kGroupWarps) * 32 + lane;
        const uint32_t bar_id = 1 + (uint32_t)grp;  // named barrier of the group's 128 threads
        const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sm);
        // Stage positions (schedule entry, item, job, stage within the item,
        // pass over the item and the item's passes).
        struct Pos {
            int k, i, jc, st, pass, np;
        };
        auto valid = [&](const Pos& q) { return q.k < sc.cnt; };
        auto at = [&](int k) {
            Pos q{k, 0, 0, 0, 0, 1};
            if constexpr (GAT) {
                for (; q.k < sc.cnt; ++q.k) {  // items of gathered jobs without live columns: skipped by every role
                    q.jc = sc.job(q.k);
                    q.np = job_passes<GAT>(p, jobs[q.jc]);
                    if (q.np > 0) break;
                }
                if (q.k < sc.cnt) q.i = sc.item(q.k);
            } else if (k < sc.cnt) {
                q.i = sc.item(k);
                q.jc = sc.job(k);
            }
            return q;
        };
        auto next = [&](Pos q) {
            if (++q.st < (int)jobs[q.jc].nst) return q;
            if constexpr (!GAT) return at(q.k + 1);
            q.st = 0;
            return ++q.pass < q.np ? q : at(q.k + 1);
        };
        auto next_own = [&](Pos q) {  // DG stages on
#pragma unroll
            for (int d = 0; d < DG; ++d)
                if (valid(q)) q = next(q);
            return q;
        };
        const Pos first = at(0);
        bool ok = true;
        // Issues stage g (at position q) of a job without a TMA map: after the
        // weight slot's previous use is released, 16-byte async copies of
        // every row's aligned segment cover, the group's 128 threads walking
        // (row, chunk) pairs chunk-fastest so a warp instruction reads a few
        // rows' contiguous bytes; one commit group per stage, empty otherwise.
        // Q4_K / Q5_K launches fetch every stage by TMA (the host builds
        // them only when every job has a tensor map): no copy path.
        constexpr bool kAllTma = TY == T_Q4_K || TY == T_Q5_K;
        auto issue = [&](const Pos& q, int g) {
            if constexpr (kAllTma) return;
            if (valid(q) && !jobs[q.jc].tma) {
                const int ws = g % SW, wu = g / SW;
                if (wu > 0 && !mbar_wait_bounded(&br.wempty[ws], (wu - 1) & 1, p.err, abort_flag, kSleepDec)) ok = false;
                const TcJob& J = jobs[q.jc];
                const int r0 = (q.i - J.item0) * kM;
                const int rows = min(kM, (int)J.n - r0);
                const int us = min(kUS, (int)J.U - kUS * q.st);
                const uint32_t segb = J.type == T_Q8_0 ? (uint32_t)us * 34u : J.seg;
                const int cpr = (int)((segb + 30) >> 4);  // chunk slots per row (>= any row's cover)
                const uint32_t dst0 = sptr(sm + p.w_off + p.w_slot * (uint32_t)ws);
                const uint8_t* src0 = J.w + (long long)r0 * J.rb + (long long)q.st * J.seg;
                for (int f = row; ok && f < rows * cpr; f += kGroupWarps * 32) {
                    const int r = f / cpr, c = f - r * cpr;
                    const uintptr_t a = (uintptr_t)(src0 + (long long)r * J.rb);
                    const uintptr_t a0 = a & ~(uintptr_t)15, a1 = (a + segb + 15) & ~(uintptr_t)15;
                    const uintptr_t off = a0 + 16 * (uintptr_t)c;
                    if (off < a1)
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst0 + (uint32_t)r * p.segp +
                                                                                       16u * (uint32_t)c),
                                     "l"(off)
                                     : "memory");
                }
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        issue(grp == 0 ? first : (valid(first) ? next(first) : first), grp);  // the group's first stage
        static_assert(DG <= 2, "a group's first stage is stage 0 or 1");
        // Stage gs's slot and earlier uses of that slot in each ring.
        int gs = 0, ws = 0, wu = 0, os = 0, ou = 0, es = 0, eu = 0;
        auto advance = [&]() {
            ++gs;
            if (++ws == SW) ws = 0, ++wu;
            if (++os == SO) os = 0, ++ou;
            if (++es == SE) es = 0, ++eu;
        };
        for (Pos cur = first; valid(cur); cur = next(cur), advance()) {
            if (gs % DG != grp) continue;  // the other group's stage
            const TcJob& J = jobs[cur.jc];
            const bool tma = kAllTma || J.tma;
            // A copied stage's group is the only one in flight.
            if (!tma) asm volatile("cp.async.wait_group 0;" ::: "memory");
            if (tma && ok && !mbar_wait_bounded(&br.wfull[ws], wu & 1, p.err, abort_flag, kSleepDec)) ok = false;
            // The A slot's previous stage is consumed (its MMAs are done), and
            // the scale slot's (its epilogue is done).
            if (ou > 0 && ok && !mbar_wait_bounded(&br.ofree[os], (ou - 1) & 1, p.err, abort_flag, kSleepDec)) ok = false;
            if (eu > 0 && ok && !mbar_wait_bounded(&br.efree[es], (eu - 1) & 1, p.err, abort_flag, kSleepDec)) ok = false;
            if (tma) {
                // The stage's weights came by TMA: each warp goes on alone.  A
                // warp that gave up keeps walking the stages without work (so
                // it still meets its group at the barriers of copied stages).
                ok = __all_sync(0xFFFFFFFFu, ok);
            } else {
                // Every thread of the group has its copies of this stage; the
                // group stops together if any of them gave up on a wait.
                uint32_t all_ok;
                asm volatile(
                    "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\t"
                    "bar.red.and.pred b, %2, 128, a;\n\tselp.u32 %0, 1, 0, b;\n\t}\n"
                    : "=r"(all_ok)
                    : "r"(ok ? 1u : 0u), "r"(bar_id)
                    : "memory");
                static_assert(kGroupWarps * 32 == 128, "a group's named barrier counts 128 threads");
                if (!all_ok) break;
            }
            if (ok) {
                const uint32_t wbase = p.w_off + p.w_slot * (uint32_t)ws, obase = p.o_off + p.o_slot * (uint32_t)os,
                               ebase = p.e_off + p.e_slot * (uint32_t)es;
                const int r0 = (cur.i - J.item0) * kM;
                const int rows = min(kM, (int)J.n - r0);
                const int us = min(kUS, (int)J.U - kUS * cur.st);
                if (row < rows) {
                    const uintptr_t a = (uintptr_t)(J.w + (long long)(r0 + row) * J.rb + (long long)cur.st * J.seg);
                    const uint32_t seg0 = tma ? wbase + (uint32_t)row * J.seg
                                                : wbase + (uint32_t)row * p.segp + (uint32_t)(a & 15);
                    const uint32_t arow = obase + (uint32_t)((row >> 3) * 256 + (row & 7) * 16);
                    const uint32_t srow = ebase + p.s_rel + (uint32_t)row * 8;
                    if constexpr (kAllTma) {  // TMA-fetched rows are 16-byte aligned
                        decode_k45_aligned<(uint32_t)TY>(sm, seg0, arow, srow);
                    } else if constexpr (TY >= 0) {
                        decode_units<(uint32_t)TY>(s32, sm, seg0, us, arow, srow);
                    } else if (J.type == T_Q4_K && (a & 15) == 0) decode_k45_aligned<T_Q4_K>(sm, seg0, arow, srow);
                    else if (J.type == T_Q5_K && (a & 15) == 0) decode_k45_aligned<T_Q5_K>(sm, seg0, arow, srow);
                    else switch (J.type) {
                        case T_Q4_K: decode_units<T_Q4_K>(s32, sm, seg0, us, arow, srow); break;
                        case T_Q5_K: decode_units<T_Q5_K>(s32, sm, seg0, us, arow, srow); break;
                        case T_Q6_K: decode_units<T_Q6_K>(s32, sm, seg0, us, arow, srow); break;
                        default: decode_units<T_Q8_0>(s32, sm, seg0, us, arow, srow); break;
                        }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // operand stores -> tensor core
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&br.afull[os]);
                    mbar_arrive(&br.sfull[es]);
                    mbar_arrive(&br.wempty[ws]);
                }
            }
            issue(next_own(cur), gs + DG);  // the group's next stage
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // no copy into shared memory outlives the role
    } else if (warp < 2 + kDecWarps + kEpiWarps) {
        // ------------------------------------------------------ epilogue --
        epilogue_role<NT, kDecWarps, GAT, TY>(sm, p, jobs, sc, br, abort_flag, tmem, warp, lane);
    } else {
        // ------------------------------------------ activation producer --
        if (lane == 0) {
            // Operand ring: activation tiles and records of each stage.
            pdl_wait();  // activations come from the quantizer grid
            int bs = 0, bu = 0, es = 0, eu = 0;  // this stage's slots, earlier uses of them
            bool ok = true;
            for (int k = 0; ok && k < sc.cnt; ++k) {
                const TcJob& J = jobs[sc.job(k)];
                const int nps = job_passes<GAT>(p, J) * (int)J.nst;
                // Pass `pass` of a gathered job reads the operand tiles of its
                // live columns [pass*N, pass*N + N): U units each.
                for (int ps = 0, st = 0, pass = 0; ps < nps; ++ps, (++st == (int)J.nst ? (st = 0, ++pass) : 0),
                         (++bs == SB ? (bs = 0, ++bu) : 0), (++es == SE ? (es = 0, ++eu) : 0)) {
                    // B slot: the MMAs of its previous stage are done; record
                    // slot: the epilogue of its previous stage is done.
                    if ((bu > 0 && !mbar_wait_bounded(&br.bfree[bs], (bu - 1) & 1, p.err, abort_flag, kSleepProd)) ||
                        (eu > 0 && !mbar_wait_bounded(&br.efree[es], (eu - 1) & 1, p.err, abort_flag, kSleepProd))) {
                        ok = false;
                        break;
                    }
                    const int us = min(kUS, (int)J.U - kUS * st);
                    const uint32_t bbytes = (uint32_t)us * J.N * 32u, dbytes = (uint32_t)us * J.N * 16u;
                    mbar_arrive_expect_tx(&br.bfull[bs], bbytes);
                    misc[kFillB + bs] += 1;
                    const size_t u0 = (size_t)pass * J.U + (size_t)kUS * st;  // first unit tile of the stage
                    bulk_g2s(sm + p.b_off + p.b_slot * (uint32_t)bs, J.act + u0 * J.N * 32, bbytes, &br.bfull[bs]);
                    mbar_arrive_expect_tx(&br.dfull[es], dbytes);
                    misc[kFillD + es] += 1;
                    bulk_g2s(sm + p.e_off + p.e_slot * (uint32_t)es + p.d_rel, J.ds + u0 * J.N * 16, dbytes,
                             &br.dfull[es]);
                }
            }
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 0) {
        // Some role gave up: let every bulk/TMA copy this CTA issued land
        // (bounded) before its shared memory is released.
        for (int s = 0; s < SW; ++s)
            if (misc[kFillW + s] > 0) mbar_wait_bounded(&br.wfull[s], (misc[kFillW + s] - 1) & 1, nullptr);
        for (int s = 0; s < SB; ++s)
            if (misc[kFillB + s] > 0) mbar_wait_bounded(&br.bfull[s], (misc[kFillB + s] - 1) & 1, nullptr);
        for (int s = 0; s < SE; ++s)
            if (misc[kFillD + s] > 0) mbar_wait_bounded(&br.dfull[s], (misc[kFillD + s] - 1) & 1, nullptr);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols)
                     : "memory");
    }
}

// ------------------------------------------------------------ host side --

uint32_t seg_bytes(uint32_t type)
{
    return type == T_Q8_0 ? (uint32_t)kUS * 34u : (uint32_t)block_bytes(type);
}

} // namespace tc

struct TcPlan {
    int device = 0;
    std::vector<tc::TcJob> jobs;
    std::vector<tc::TcQTask> tasks;
    tc::TcParams pp{};
    tc::TcQParams qp{};
    int grid = 0;
    size_t smem = 0;
    tc::TcJob* d_jobs = nullptr;
    tc::TcQTask* d_tasks = nullptr;
    uint32_t* d_sched = nullptr;
    int* d_sched_off = nullptr;
    uint8_t* d_act = nullptr;
    int bmax = 1;  // most tokens of any job: selects the epilogue's tokens per thread
    int ty = -1;   // the weight type every job shares (kernel specialised to it), -1 if mixed
};

int tc_plan_create(const GemvJobIn* in, int njobs, TcPlan** out)
{
    using namespace tc;
    if (!out || !in || njobs <= 0 || njobs > kTcMaxJobs) return QUANTR_ERR_BAD_ARG;
    *out = nullptr;
    TcPlan* P = new (std::nothrow) TcPlan();
    if (!P) return QUANTR_ERR_OOM;
    cudaGetDevice(&P->device);
    // Activation tasks, one per distinct (x, ldx, d, B, element order); the
    // operand layout depends on the weight type only through that order.
    std::map<std::tuple<const float*, const float*, long long, int, int, int>, int> dedupe;
    size_t act_total = 0;
    long long blocks = 0;
    int Nmax = 16, Bmax = 1, item = 0;
    bool gathered = false;
    std::vector<size_t> task_act_off;
    std::vector<int> job_task;
    for (int j = 0; j < njobs; ++j) {
        const GemvJobIn& a = in[j];
        if (!type_supported(a.type) || a.type == T_F32) {
            delete P;
            return QUANTR_ERR_UNSUPPORTED_TYPE;
        }
        const bool pre = a.act != nullptr;  // activations given as operand tiles
        if (!a.w || (!pre && (!a.x || a.ldx < a.d)) || (pre && !a.ds) ||
            (a.g_counts && (!a.g_offsets || !a.g_list || a.g_e < 0 || !pre || a.B != 16)) || !a.out || a.n <= 0 ||
            a.B <= 0 || a.B > kMaxN || a.ldo < a.n ||
            ((uintptr_t)a.w & 15) || row_bytes(a.type, a.d) <= 0) {
            delete P;
            return QUANTR_ERR_BAD_ARG;
        }
        TcJob J{};
        J.w = a.w;
        J.rb = row_bytes(a.type, a.d);
        J.type = a.type;
        J.n = (uint32_t)a.n;
        J.U = (uint32_t)((a.d / block_elems(a.type)) * block_units(a.type));
        J.B = (uint32_t)a.B;
        J.N = (uint32_t)std::max(16, (a.B + 15) / 16 * 16);
        J.nst = (J.U + kUS - 1) / kUS;
        J.seg = seg_bytes(a.type);
        // D s32 (bits 4-5 = 2); A unsigned 8-bit for the K-quants (0..63),
        // signed for Q8_0 (bit 7); B signed (bit 10); K-major A and B;
        // N >> 3 at bit 17; M >> 4 at bit 24.
        J.idesc = (2u << 4) | ((a.type == T_Q8_0 ? 1u : 0u) << 7) | (1u << 10) | ((J.N >> 3) << 17) |
                  ((uint32_t)(kM >> 4) << 24);
        J.out = a.out;
        J.ldo = a.ldo;
        J.tiles = (a.n + kM - 1) / kM;
        J.item0 = item;
        item += J.tiles;
        Nmax = std::max(Nmax, (int)J.N);
        Bmax = std::max(Bmax, a.B);
        J.ge = -1;
        if (a.g_counts) {  // every gathered job of a launch shares one set of counts and lists
            TcParams& q = P->pp;
            if (gathered && (a.g_counts != q.gcounts || a.g_offsets != q.goffsets || a.g_list != q.glist)) {
                delete P;
                return QUANTR_ERR_BAD_ARG;
            }
            gathered = true;
            q.gcounts = a.g_counts;
            q.goffsets = a.g_offsets;
            q.glist = a.g_list;
            J.ge = a.g_e;
        }
        if (pre) {
            J.act = a.act;
            J.ds = a.ds;
            job_task.push_back(-1);
            P->jobs.push_back(J);
            continue;
        }
        const int perm = a.type == T_Q8_0 ? 0 : (a.type == T_Q6_K ? 2 : 1);
        auto key = std::make_tuple(a.x, a.xmul, a.ldx, a.d, a.B, perm);
        auto it = dedupe.find(key);
        int ti;
        if (it == dedupe.end()) {
            TcQTask t{};
            t.x = a.x;
            t.xmul = a.xmul;
            t.ldx = a.ldx;
            t.U = (int)J.U;
            t.B = a.B;
            t.N = (int)J.N;
            t.type = (int)a.type;
            t.vec = ((uintptr_t)a.x % 16 == 0 && a.ldx % 4 == 0) ? 1 : 0;
            t.blk0 = blocks;
            blocks += (long long)a.B * J.U;
            task_act_off.push_back(act_total);
            act_total += ((size_t)J.U * J.N * 48 + 255) & ~size_t(255);
            ti = (int)P->tasks.size();
            P->tasks.push_back(t);
            dedupe[key] = ti;
        } else {
            ti = it->second;
        }
        job_task.push_back(ti);
        P->jobs.push_back(J);
    }
    if (item >= (1 << 20)) {  // schedule entries hold the item in 20 bits
        delete P;
        return QUANTR_ERR_TOO_LARGE;
    }
    // Static schedule: items (128-row tiles, J.nst stages each) dealt longest
    // first to the least-loaded CTA (ties to the lower index), so every CTA
    // ends within one item's stages of the others; entries (job << 20) | item.
    const int grid = std::min(device_sm_count(), item);
    std::vector<std::vector<uint32_t>> lists((size_t)grid);
    {
        std::vector<std::pair<int, uint32_t>> order;  // (-stages, entry)
        order.reserve((size_t)item);
        for (size_t j = 0; j < P->jobs.size(); ++j)
            for (uint32_t t = 0; t < P->jobs[j].tiles; ++t)
                order.push_back({-(int)P->jobs[j].nst, ((uint32_t)j << 20) | (P->jobs[j].item0 + t)});
        std::stable_sort(order.begin(), order.end(),
                         [](const std::pair<int, uint32_t>& a, const std::pair<int, uint32_t>& b) {
                             return a.first < b.first;
                         });
        std::priority_queue<std::pair<long long, int>, std::vector<std::pair<long long, int>>,
                            std::greater<std::pair<long long, int>>>
            load;
        for (int c = 0; c < grid; ++c) load.push({0LL, c});
        for (const auto& o : order) {
            auto top = load.top();
            load.pop();
            lists[(size_t)top.second].push_back(o.second);
            load.push({top.first - o.first, top.second});
        }
    }
    std::vector<uint32_t> sched;
    std::vector<int> sched_off(1, 0);
    size_t maxcnt = 0;
    for (const auto& l : lists) {
        sched.insert(sched.end(), l.begin(), l.end());
        sched_off.push_back((int)sched.size());
        maxcnt = std::max(maxcnt, l.size());
    }
    TcParams& pp = P->pp;
    // 2-D TMA maps for the jobs whose rows are 16-byte aligned (Q4_K, Q5_K);
    // the others (and all jobs, if the driver entry point is unavailable)
    // keep the per-thread async copies.
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static bool looked_up = false;
    if (!looked_up) {
        looked_up = true;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&encode, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            encode = nullptr;
        cudaGetLastError();
    }
    uint32_t seg_tma = 0, seg_copy = 0;  // widest stage segment of the TMA jobs and of the copied jobs
    for (size_t j = 0; j < P->jobs.size(); ++j) {
        TcJob& J = P->jobs[j];
        J.tma = 0;
        if (encode && (J.type == T_Q4_K || J.type == T_Q5_K) && (J.rb % 16) == 0) {
            const cuuint64_t dims[2] = {(cuuint64_t)J.rb, (cuuint64_t)J.n};
            const cuuint64_t strides[1] = {(cuuint64_t)J.rb};
            const cuuint32_t box[2] = {J.seg, (cuuint32_t)kM};
            const cuuint32_t estr[2] = {1, 1};
            if (encode(&pp.tmap[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(J.w), dims, strides, box,
                       estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
                J.tma = 1;
        }
        if (J.tma) seg_tma = std::max(seg_tma, J.seg);
        else seg_copy = std::max(seg_copy, J.seg);
    }
    // Shared memory: barriers | SW weight slots | SO A-tile slots | SB B-tile
    // slots | SE epilogue slots of {records | scales} | job table | this CTA's
    // schedule.  A TMA job's stage lands as 128 rows x seg bytes; a copied
    // job's row is the 16-byte aligned cover of its segment (up to 15 bytes
    // before and 15 after, plus one word the decoder may read past).
    const uint32_t segp = seg_copy ? (seg_copy + 45) & ~15u : 16u;
    const uint32_t wslot = (std::max(kM * (seg_copy ? segp : 0u), kM * seg_tma) + 1023) & ~1023u;
    const uint32_t abytes = kUS * kATile, bbytes = kUS * (uint32_t)Nmax * 32u, dbytes = kUS * (uint32_t)Nmax * 16u,
                   sbytes = kUS * kM * 8u;
    const uint32_t oslot = abytes, bslot = (bbytes + 1023) & ~1023u, eslot = (dbytes + sbytes + 127) & ~127u;
    const uint32_t bars = 1024, tbl = ((uint32_t)(P->jobs.size() * sizeof(TcJob)) + 127) & ~127u;
    const uint32_t stbl = ((uint32_t)(maxcnt * 4) + 127) & ~127u;
    const int SO = kMaxSO;
    // Deep B-tile and epilogue rings (activations are fetched that many
    // stages ahead; the epilogue may trail the decoders by SE stages) as long
    // as three weight slots remain; at least two of each.
    int SB = 4, SE = kMaxSE, SW = 0;
    for (;;) {
        const long long room = (long long)kSmemMax - bars - tbl - stbl - (long long)SO * oslot -
                               (long long)SB * bslot - (long long)SE * eslot;
        SW = room > 0 ? (int)std::min<long long>(kMaxSW, room / wslot) : 0;
        if (SW >= 3 || (SB == 2 && SE == 2)) break;
        if (SB > 2) --SB;
        if (SE > 2) --SE;
    }
    if (SW < 2) {
        delete P;
        return QUANTR_ERR_TOO_LARGE;
    }
    pp.njobs = (int)P->jobs.size();
    pp.total_items = item;
    pp.SW = (uint32_t)SW;
    pp.SO = (uint32_t)SO;
    pp.SB = (uint32_t)SB;
    pp.SE = (uint32_t)SE;
    pp.ncol = (uint32_t)Nmax;
    pp.gathered = gathered ? 1 : 0;
    P->bmax = Bmax;
    P->ty = (int)P->jobs[0].type;
    for (const auto& J : P->jobs)  // a Q4_K/Q5_K kernel assumes every job has a tensor map
        if ((int)J.type != P->ty || ((J.type == T_Q4_K || J.type == T_Q5_K) && !J.tma)) P->ty = -1;
    pp.NB = (uint32_t)std::min(kMaxNB, 512 / (kUS * Nmax));  // 4, 2 or 1 stage buffers for N = 16, 32, 64
    uint32_t cols = 32;
    while (cols < pp.NB * kUS * pp.ncol) cols <<= 1;
    pp.tmem_cols = cols;
    pp.segp = segp;
    pp.w_off = bars;
    pp.w_slot = wslot;
    pp.o_off = bars + (uint32_t)SW * wslot;
    pp.o_slot = oslot;
    pp.b_off = pp.o_off + (uint32_t)SO * oslot;
    pp.b_slot = bslot;
    pp.e_off = pp.b_off + (uint32_t)SB * bslot;
    pp.e_slot = eslot;
    pp.d_rel = 0;
    pp.s_rel = dbytes;
    pp.jobs_off = pp.e_off + (uint32_t)SE * eslot;
    pp.sched_smem = pp.jobs_off + tbl;
    P->smem = pp.sched_smem + stbl;
    P->grid = grid;

    cudaError_t e = cudaMalloc((void**)&P->d_act, std::max<size_t>(act_total, 256));
    if (e == cudaSuccess) e = cudaMemset(P->d_act, 0, std::max<size_t>(act_total, 256));  // padding tokens stay 0
    if (e == cudaSuccess) {
        for (size_t t = 0; t < P->tasks.size(); ++t) {
            P->tasks[t].act = P->d_act + task_act_off[t];
            P->tasks[t].ds = P->tasks[t].act + (size_t)P->tasks[t].U * P->tasks[t].N * 32;
        }
        for (size_t j = 0; j < P->jobs.size(); ++j) {
            if (job_task[j] < 0) continue;  // operand tiles given
            P->jobs[j].act = P->tasks[job_task[j]].act;
            P->jobs[j].ds = P->tasks[job_task[j]].ds;
        }
    }
    if (e == cudaSuccess) e = cudaMalloc((void**)&P->d_jobs, P->jobs.size() * sizeof(TcJob));
    if (e == cudaSuccess)
        e = cudaMemcpy(P->d_jobs, P->jobs.data(), P->jobs.size() * sizeof(TcJob), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && !P->tasks.empty())  // none when every job came with operand tiles
        e = cudaMalloc((void**)&P->d_tasks, P->tasks.size() * sizeof(TcQTask));
    if (e == cudaSuccess && !P->tasks.empty())
        e = cudaMemcpy(P->d_tasks, P->tasks.data(), P->tasks.size() * sizeof(TcQTask), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc((void**)&P->d_sched, sched.size() * sizeof(uint32_t));
    if (e == cudaSuccess)
        e = cudaMemcpy(P->d_sched, sched.data(), sched.size() * sizeof(uint32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc((void**)&P->d_sched_off, sched_off.size() * sizeof(int));
    if (e == cudaSuccess)
        e = cudaMemcpy(P->d_sched_off, sched_off.data(), sched_off.size() * sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        const int code = e == cudaErrorMemoryAllocation ? QUANTR_ERR_OOM : QUANTR_ERR_CUDA;
        cudaGetLastError();
        tc_plan_destroy(P);
        return code;
    }
    pp.jobs = P->d_jobs;
    pp.sched = P->d_sched;
    pp.sched_off = P->d_sched_off;
    P->qp.tasks = P->d_tasks;
    P->qp.ntasks = (int)P->tasks.size();
    P->qp.total = blocks;
    *out = P;
    return QUANTR_OK;
}

namespace tc {

template <int DG, int EG, int NT, bool GAT, int TY>
cudaError_t launch_tc_k(const TcPlan* P, const TcParams& pp, const LaunchCfg& c)
{
    static int configured = -1;
    cudaError_t e = ensure_smem_attr(&k_tc_program<DG, EG, NT, GAT, TY>, (int)kSmemMax, configured);
    if (e != cudaSuccess) return e;
    return launch_ex(&k_tc_program<DG, EG, NT, GAT, TY>, dim3(P->grid), dim3(Split<DG, EG>::threads), P->smem, c,
                     pp);
}

template <int DG, int EG, int NT, bool GAT>
cudaError_t launch_tc_t(const TcPlan* P, const TcParams& pp, const LaunchCfg& c)
{
    // Measured on B200: batch 4 64 -> 61 us per c2 step, batch 16 97 -> 87 us,
    // the c4 MoE layer 341 -> 328 us.
    switch (P->ty) {
    case T_Q4_K: return launch_tc_k<DG, EG, NT, GAT, T_Q4_K>(P, pp, c);
    case T_Q5_K: return launch_tc_k<DG, EG, NT, GAT, T_Q5_K>(P, pp, c);
    case T_Q6_K: return launch_tc_k<DG, EG, NT, GAT, T_Q6_K>(P, pp, c);
    case T_Q8_0: return launch_tc_k<DG, EG, NT, GAT, T_Q8_0>(P, pp, c);
    default: return launch_tc_k<DG, EG, NT, GAT, -1>(P, pp, c);
    }
}

template <int DG, int EG, int NT>
cudaError_t launch_tc(const TcPlan* P, const TcParams& pp, const LaunchCfg& c)
{
    // Gathered jobs (MoE experts) always run 16 columns: only that split is built for them.
    if constexpr (DG == 2 && EG == 2 && NT == 8)
        if (pp.gathered) return launch_tc_t<DG, EG, NT, true>(P, pp, c);
    if (pp.gathered) return cudaErrorNotSupported;
    return launch_tc_t<DG, EG, NT, false>(P, pp, c);
}

} // namespace tc

cudaError_t tc_plan_run(TcPlan* P, int* err, cudaStream_t stream)
{
    using namespace tc;
    LaunchCfg c;
    c.stream = stream;
    if (P->qp.total > 0) {  // no quantizer when every job came with operand tiles
        const long long qgrid =
            std::max(1LL, std::min<long long>((P->qp.total + 255) / 256, 8LL * device_sm_count()));
        const cudaError_t e = launch_ex(&k_tc_quant, dim3((unsigned)qgrid), dim3(256), 0, c, P->qp);
        if (e != cudaSuccess) return e;
    }
    TcParams pp = P->pp;
    pp.err = err;
    // The split and the epilogue's tokens per thread (see Split).
    if (P->bmax <= 1) return launch_tc<2, 1, 1>(P, pp, c);
    if (P->bmax <= 2) return launch_tc<2, QR_TC_B4_EG, 2 / QR_TC_B4_EG>(P, pp, c);
    if (P->bmax <= 4) return launch_tc<2, QR_TC_B4_EG, 4 / QR_TC_B4_EG>(P, pp, c);
    if (P->bmax <= 8) return launch_tc<2, QR_TC_B8_EG, 8 / QR_TC_B8_EG>(P, pp, c);
    if (pp.ncol <= 16) return launch_tc<QR_TC_N16_DG, QR_TC_N16_EG, 16 / QR_TC_N16_EG>(P, pp, c);
    if (pp.ncol == 32) return launch_tc<1, 4, 8>(P, pp, c);
    return launch_tc<1, 4, 16>(P, pp, c);
}

void tc_split_narrow(std::vector<GemvJobIn>& tcj, int sms)
{
    auto tiles = [&]() {
        long long t = 0;
        for (const auto& g : tcj) t += (g.n + 127) / 128;
        return t;
    };
    while (!tcj.empty() && tiles() < sms && tcj.size() < (size_t)kTcMaxJobs) {
        size_t wi = 0;
        for (size_t i = 1; i < tcj.size(); ++i)
            if (tcj[i].B > tcj[wi].B) wi = i;
        if (tcj[wi].B <= 16 || tcj[wi].g_counts) break;
        GemvJobIn hi = tcj[wi];
        const int keep = ((tcj[wi].B / 2 + 15) / 16) * 16;
        tcj[wi].B = keep;
        hi.B -= keep;
        hi.x += (long long)keep * hi.ldx;
        hi.out += (long long)keep * hi.ldo;
        if (hi.xmul) hi.xmul += (long long)keep * hi.ldx;
        tcj.push_back(hi);
    }
}

cudaError_t launch_gemv_tc(const uint8_t* w, uint32_t type, int n, int d, int B, const float* x, long long ldx,
                           float* out, long long ldo, int* err, cudaStream_t stream)
{
    if (B < 2 || n <= 0 || !x || !out || ldx < d || ldo < n || ((uintptr_t)w & 15) ||
        !(type == T_Q8_0 || type == T_Q4_K || type == T_Q5_K || type == T_Q6_K) || row_bytes(type, d) <= 0)
        return cudaErrorNotSupported;
    int dev = 0;
    cudaGetDevice(&dev);
    using Key = std::tuple<int, const uint8_t*, uint32_t, int, int, int, const float*, long long, float*, long long>;
    static std::mutex mu;
    static std::map<Key, std::vector<TcPlan*>> cache;
    std::lock_guard<std::mutex> lk(mu);  // held while the plans are enqueued
    const Key key{dev, w, type, n, d, B, x, ldx, out, ldo};
    auto it = cache.find(key);
    if (it == cache.end()) {
        if (cache.size() >= 64) {  // bounded: drop every plan (tc_plan_destroy synchronises the device)
            for (auto& kv : cache)
                for (TcPlan* p : kv.second) tc_plan_destroy(p);
            cache.clear();
        }
        std::vector<GemvJobIn> jobs;
        for (int b0 = 0; b0 < B; b0 += kTcMaxB)
            jobs.push_back(GemvJobIn{w, type, n, d, std::min(kTcMaxB, B - b0), x + (long long)b0 * ldx, ldx,
                                     out + (long long)b0 * ldo, ldo});
        tc_split_narrow(jobs, device_sm_count());
        std::vector<TcPlan*> plans;
        for (size_t j0 = 0; j0 < jobs.size(); j0 += kTcMaxJobs) {
            TcPlan* p = nullptr;
            if (tc_plan_create(jobs.data() + j0, (int)std::min<size_t>(kTcMaxJobs, jobs.size() - j0), &p) != 0) {
                for (TcPlan* q : plans) tc_plan_destroy(q);
                plans.clear();
                cudaGetLastError();
                break;
            }
            plans.push_back(p);
        }
        it = cache.emplace(key, std::move(plans)).first;
    }
    if (it->second.empty()) return cudaErrorNotSupported;
    for (TcPlan* p : it->second) {
        const cudaError_t e = tc_plan_run(p, err, stream);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

void tc_plan_destroy(TcPlan* P)
{
    if (!P) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(P->device);
    cudaDeviceSynchronize();
    cudaFree(P->d_jobs);
    cudaFree(P->d_tasks);
    cudaFree(P->d_act);
    cudaFree(P->d_sched);
    cudaFree(P->d_sched_off);
    if (prev >= 0) cudaSetDevice(prev);
    delete P;
}

void tc_plan_info(const TcPlan* P, int* items, int* grid, int* smem)
{
    if (items) *items = P->pp.total_items;
    if (grid) *grid = P->grid;
    if (smem) *smem = (int)P->smem;
}

} // namespace qr
