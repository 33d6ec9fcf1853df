// step_kernel.cu - the persistent decode step: one cooperative launch per
// decode token instead of one launch per op.
//
// LMc's model_forward (src/ops.c:212-237, src/ops_llama.c:157-192) is a fixed
// sequence of matmul_vec / attention / norm calls.  Launched one kernel per
// op, a GPT-2 Small decode step is 63 launches, and at batch 1 every launch
// pays a fixed cost (the previous kernel draining, the next one's CTAs
// starting, its activation setup) several times larger than the time its
// weights take to stream.  Here the host encodes the step once as a list of
// ops; one CTA-resident grid (co-residency guaranteed by the cooperative
// launch) walks the list, every CTA doing its share of each op, and the CTAs
// meet at a grid-wide barrier between dependent ops: a counter in device
// memory (release add, acquire poll, bounded by %globaltimer), ~1 us instead
// of a kernel boundary.
//
// Weights never depend on activations, so a warp that has finished its units
// of one GEMV immediately starts the bulk copies of its first units of the
// NEXT GEMV into its ring (shared memory at a fixed offset, slots sized for
// the largest unit), and asks L2 for the units after those; the copies land
// while the CTA waits at the barrier, runs attention, and builds the next
// activation fragments.  The GEMV, attention and embedding bodies are the
// same device code as the standalone kernels (tiled_gemv.cuh, attention.cuh,
// lmc_blocks.cuh), so results match them; only activations written earlier in
// the same launch are read through L2 (ld.cg).
//
// Limits (the host falls back to the per-op launches otherwise): one GPU (no
// collective inside), batch <= 2, every GEMV on the tiled tensor-core layout,
// attention with head size 64 or 128 and in-launch split merging, embedding types Q4_K/Q6_K/Q8_0/F16/
// F32.  A barrier or ring wait that runs out sets an abort flag that every
// CTA polls; all CTAs then drain their copies and return, and
// lmc_step_status() reports LMC_ERR_TIMEOUT and resets the barrier state.
#include "attention.cuh"
#include "sample.cuh"
#include "tiled_gemv.cuh"

#include <stdlib.h>

#include <mutex>
#include <vector>

namespace {

constexpr int SLOT = Q80_UNIT;  // ring slot bytes: the largest unit

struct EmbedArgs {
    const uint8_t *wte;
    const float *wpe;
    const int *tok, *pos;
    int D, V, S, type;
    float *out;
    double *stats_out;  // {sum x, sum x^2} per row for the norm that reads x, or NULL
};
// The K/V rows an attention op will read (positions 0..pos-1 of every
// sequence and kv head): asked of L2 by the GEMV op before it.
struct KvPf {
    const uint8_t *kc, *vc;
    const int *pos;
    int Hkv, S, row_bytes, nb;
};
struct AdvArgs {
    unsigned long long *keys;
    int *next, *tok, *pos, *step, *ids;
    int *next_host;  // KEYS: the picks also written here (mapped host memory), or NULL
    const int *prompt;
    int n_prompt, n_new, generate, from_next;
};
struct SampArgs {
    const float *logits;
    int V;
    float temperature, top_p;
    unsigned long long *rng;
    int *next;
    const int *step;
    int n_prompt;
};
struct alignas(16) DOp {
    int kind, sync, nb;
    int qt;           // GEMV: 4 / 6 / 8
    int next_gemv;    // index of the next GEMV op (its ring is filled at the end of this one), -1 none
    int nqt;          // its format
    int kv, dh;       // ATTN: cache rows LMC_KV_F32 / F16 / Q8; head size 64 / 128
    int items;        // ATTN: splits x kv heads x batch
    int kpf;          // GEMV: 1 = prefetch kp into L2 first
    int ff;           // GEMV: 1 = the latency (fp32) form, 0 = the tensor-core form
    TArgs g;
    TArgs ng;         // the next GEMV's arguments (its ring prefill reads them here)
    KvPf kp;
    AttnArgs at;
    EmbedArgs e;
    AdvArgs v;
    SampArgs sm;
};
// Barrier arrivals go to BAR_GROUPS counters (CTA c to counter c % BAR_GROUPS),
// each on its own 128-byte line, so the atomics do not queue on one address.
constexpr int BAR_GROUPS = 8;
struct alignas(128) BarCount {
    unsigned v;
};
struct StepCtl {
    BarCount cnt[BAR_GROUPS];   // arrivals, never reset between launches
    unsigned base[BAR_GROUPS];  // each counter at the start of the next launch
    int abort;                  // set when a wait ran out: every CTA leaves
    int where;                  // op index + 1 of the wait that ran out
};
// A byte range asked of L2 at the start of a step: 16-byte aligned start and
// length (the norm weights and biases of every GEMV, which are otherwise
// first read from HBM on the critical path of their op).
struct PfRange {
    const void *p;
    unsigned bytes;
};
struct StepParams {
    const DOp *ops;
    int nops, first_gemv, ring_off, stages;
    StepCtl *ctl;
    double *stats;  // norm statistics slots, zeroed again at the end of each launch
    int stats_n;    // doubles in the slots
    const PfRange *pf;
    int pf_n;
    // Tokens and positions passed with the launch (lmc_step_prog_launch_imm):
    // CTA b stores row b's into tok_dst / pos_dst before its first op (the
    // embedding, which CTA b runs); every other reader comes after a barrier.
    int imm_n, imm_tok[2], imm_pos[2];
    int *tok_dst, *pos_dst;
};

__device__ long long g_step_wait_ns = 1000000000ll;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Arrivals the counter of group k holds after `passed` barriers of a launch
// that started at base[k]: CTAs c with c % BAR_GROUPS == k arrive there.
__device__ __forceinline__ unsigned group_size(int k) {
    return (gridDim.x + BAR_GROUPS - 1 - (unsigned)k) / BAR_GROUPS;
}

// Grid-wide barrier in two phases.  grid_arrive: once every thread of the
// CTA is done with the op (bar.sync), thread 0 adds its arrival to its
// group's counter with release semantics.  Work that the
// next op does not read (the next GEMV's weight copies, K/V prefetch) runs
// between the phases.  grid_wait: lanes 0..7 of warp 0 poll one counter each
// until every group is complete, the abort flag is set, or the wait limit
// passes (then they set the flag); meanwhile the other warps copy the next op
// into `next_op` (the op list is constant).  Returns false when the CTA must
// leave.
// The arrival is one release add: the CTA barrier before it orders every
// thread's writes before thread 0's release, and release is cumulative, so no
// separate fence (a second round trip to L2) is needed.  Likewise the
// pollers' acquire loads plus the CTA barrier after them order every thread's
// later reads.
__device__ __forceinline__ void grid_arrive(StepCtl *ctl) {
    __syncthreads();
    if (threadIdx.x == 0)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&ctl->cnt[blockIdx.x % BAR_GROUPS].v)
                     : "memory");
}
__device__ __forceinline__ bool grid_wait(StepCtl *ctl, const unsigned *base, unsigned passed, int where, int *sh_ok,
                                          const DOp *next_src, DOp *next_op) {
    const int lane = threadIdx.x & 31;
    if (threadIdx.x < 32) {
        const int k = lane < BAR_GROUPS ? lane : 0;
        const unsigned target = base[k] + passed * group_size(k);
        int ok = 1;
        long long t0 = 0;
        for (unsigned it = 0;; it++) {
            const bool mine = lane >= BAR_GROUPS || (int)(ld_acquire_u32(&ctl->cnt[k].v) - target) >= 0;
            if (__all_sync(0xffffffffu, mine)) break;
            if ((it & 31) == 31) {
                int stop = 0;
                if (lane == 0) {
                    if (*(volatile int *)&ctl->abort) {
                        stop = 1;
                    } else {
                        const long long t = globaltimer_ns();
                        if (!t0) t0 = t;
                        else if (t - t0 > g_step_wait_ns) {
                            atomicExch(&ctl->where, where + 1);
                            atomicExch(&ctl->abort, 1);
                            stop = 1;
                        }
                    }
                }
                if (__shfl_sync(0xffffffffu, stop, 0)) {
                    ok = 0;
                    break;
                }
            }
        }
        if (lane == 0) *sh_ok = ok;
    } else if (next_src) {
        const int4 *src = reinterpret_cast<const int4 *>(next_src);
        int4 *dst = reinterpret_cast<int4 *>(next_op);
        for (int w = threadIdx.x - 32; w < (int)(sizeof(DOp) / 16); w += NTHR - 32) dst[w] = __ldg(src + w);
    }
    __syncthreads();
    return *sh_ok != 0;
}
__device__ __forceinline__ bool grid_sync(StepCtl *ctl, const unsigned *base, unsigned passed, int where, int *sh_ok,
                                          const DOp *next_src, DOp *next_op) {
    grid_arrive(ctl);
    return grid_wait(ctl, base, passed, where, sh_ok, next_src, next_op);
}

// Per-warp bulk-copy ring, carried across the GEMV ops of the step: the next
// slot to consume, its phase parity, and the copies issued but not consumed.
struct Ring {
    uint8_t *slots;
    uint64_t *bars;
    int stages, s, inflight;
    uint32_t par;
};

// Units [w0, w1) of the row tiles [t0, t1) of this CTA for warp `wid`; false
// when the CTA has no row tile in this GEMV.
__device__ __forceinline__ bool warp_units(const TArgs &a, int cid, int wid, int &w0, int &w1, int &t0, int &t1) {
    if (cid >= a.NC) {
        w0 = w1 = t0 = t1 = 0;
        return false;
    }
    // 32-bit products: cid * RT < 2^31 for every shape the host plans here;
    // (gate, up) tile pairs stay in one CTA
    if (a.epi & LMC_EPI_GLU_PAIRS) {
        t0 = 2 * (cid * (a.RT >> 1) / a.NC);
        t1 = 2 * ((cid + 1) * (a.RT >> 1) / a.NC);
    } else {
        t0 = cid * a.RT / a.NC;
        t1 = (cid + 1) * a.RT / a.NC;
    }
    const int Uc = (t1 - t0) * a.KB;
    w0 = Uc * wid / WARPS;
    w1 = Uc * (wid + 1) / WARPS;
    return true;
}

// Start the copies of this warp's first units of GEMV `a` into its ring, and
// ask L2 for the next `pf` units after those.
__device__ __forceinline__ void ring_prefill(Ring &r, const TArgs &a, int qt, int lane, int wid) {
    int w0, w1, t0, t1;
    if (!warp_units(a, blockIdx.x, wid, w0, w1, t0, t1) || w1 <= w0) return;
    const int unit = unit_bytes(qt);
    const uint8_t *wbase = a.w + (size_t)t0 * a.KB * unit;
    const int n = min(r.stages, w1 - w0);
    if (lane == 0) {
        int s = r.s;
        for (int k = 0; k < n; k++) {
            issue_unit(&r.bars[s], r.slots + (size_t)s * SLOT, wbase + (size_t)(w0 + k) * unit, (uint32_t)unit);
            if (++s == r.stages) s = 0;
        }
        const int p1 = min(w1, w0 + r.stages + a.pf);
        for (int q = w0 + r.stages; q < p1; q++) prefetch_l2(wbase + (size_t)q * unit, (uint32_t)unit);
    }
    r.inflight += n;
    __syncwarp();
}

// Ask L2 for the K/V rows the coming attention op reads (positions 0..pos-1
// of each sequence and kv head; the rows were written by earlier steps), in
// 16 KB pieces, one (sequence, kv head, K or V) range per CTA.  Issued by
// warp 1, so that warp 0 (the barrier's poller) is not held up.
__device__ __forceinline__ void kv_prefetch(const KvPf &k) {
    if (threadIdx.x != 32) return;
    const int items = k.nb * k.Hkv * 2;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int half = it & 1, bh = it >> 1, b = bh / k.Hkv, kh = bh % k.Hkv;
        const int pos = min(max(__ldcg(k.pos + b), 0), k.S);
        const uint8_t *base = (half ? k.vc : k.kc) + ((size_t)b * k.Hkv + kh) * k.S * (size_t)k.row_bytes;
        const size_t bytes = (size_t)pos * k.row_bytes;
        for (size_t o = 0; o < bytes; o += 16384)
            prefetch_l2(base + o, (uint32_t)min((size_t)16384, bytes - o));
    }
}

// The output of this lane in one row tile (batch <= 2, so a tile has at most
// 32 outputs: lane = 16 * batch row + tile row): bias (preloaded in pbias when
// given), GELU, residual add (the old value preloaded in `pre` when given),
// the greedy-pick key, and the sums of the final values for the norm that
// reads them next.
__device__ __forceinline__ void step_epilogue_tile(const TArgs &a, int row0, const float *ar, int lane,
                                                   unsigned long long &best, const float *pre, const float *pbias,
                                                   double (&st)[2]) {
    const int b = lane >> 4, row = row0 + (lane & 15);
    if (b >= a.nb || row >= a.M) return;
    float v = ar[lane];
    if (a.bias) v += pbias ? *pbias : __ldg(a.bias + row);
    if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
    float *o = a.y + (size_t)b * a.ldy + row;
    const float out = (a.epi & LMC_EPI_ACCUM) ? (pre ? *pre : __ldcg(o)) + v : v;
    *o = out;
    const unsigned long long k = lmc_argmax_key(v, row + a.key_base);
    best = k > best ? k : best;
    st[0] += (double)out;
    st[1] += (double)out * (double)out;
}

// the latency GEMV's unit bodies (inside this file's anonymous namespace)
#include "ff_unit.cuh"

// x after its prologue, as fp32 rows xs[b][K] at shared-memory offset 0 (one
// trip to L2: the norm statistics come from the op that wrote x).
__device__ __forceinline__ void load_x_f32(float *xs, float *mr, const TArgs &a) {
    const int K = a.KB * 256, tid = threadIdx.x;
    float *mean = mr, *rstd = mr + 2;
    const bool ln = a.pro == LMC_PRO_LAYERNORM;
    if ((ln || a.pro == LMC_PRO_RMSNORM) && K <= NTHR * 4) {
        // rows of at most one float4 per thread: the x, weight and bias loads
        // are issued before the statistics are waited for (one trip to L2)
        const int k = tid * 4;
        const bool act = k < K;
        float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0, w = v0, c = v0;
        if (act) {
            v0 = __ldcg(reinterpret_cast<const float4 *>(a.x + k));
            if (a.nb > 1) v1 = __ldcg(reinterpret_cast<const float4 *>(a.x + a.ldx + k));
            w = __ldg(reinterpret_cast<const float4 *>(a.pw + k));
            if (ln) c = __ldg(reinterpret_cast<const float4 *>(a.pb + k));
        }
        if (tid < a.nb) {
            const double sx = __ldcg(a.stats + 2 * tid), sq = __ldcg(a.stats + 2 * tid + 1);
            const double mu = ln ? sx / (double)K : 0.0;
            const double var = fmax(sq / (double)K - mu * mu, 0.0);
            mean[tid] = (float)mu;
            rstd[tid] = 1.0f / sqrtf((float)var + (ln ? 1e-5f : a.eps));
        }
        __syncthreads();
        if (act) {
#pragma unroll
            for (int b = 0; b < 2; b++) {
                if (b >= a.nb) break;
                const float4 v = b ? v1 : v0;
                const float m = mean[b], r = rstd[b];
                const float4 o = ln ? make_float4((v.x - m) * r * w.x + c.x, (v.y - m) * r * w.y + c.y,
                                                  (v.z - m) * r * w.z + c.z, (v.w - m) * r * w.w + c.w)
                                    : make_float4(w.x * r * v.x, w.y * r * v.y, w.z * r * v.z, w.w * r * v.w);
                *reinterpret_cast<float4 *>(xs + b * K + k) = o;
            }
        }
        __syncthreads();
        return;
    }
    if (a.pro == LMC_PRO_LAYERNORM || a.pro == LMC_PRO_RMSNORM) {
        if (tid < a.nb) {
            const double sx = __ldcg(a.stats + 2 * tid), sq = __ldcg(a.stats + 2 * tid + 1);
            const double mu = a.pro == LMC_PRO_RMSNORM ? 0.0 : sx / (double)K;
            const double var = fmax(sq / (double)K - mu * mu, 0.0);
            mean[tid] = (float)mu;
            rstd[tid] = 1.0f / sqrtf((float)var + (a.pro == LMC_PRO_RMSNORM ? a.eps : 1e-5f));
        }
        __syncthreads();
    }
    const XView<true> xv{a.x, a.x2, a.pw, a.pb, a.ldx, a.pro, mean, rstd};
    for (int b = 0; b < a.nb; b++) {
        int k = tid * 4;
        for (; k + 3 * NTHR * 4 < K; k += 4 * NTHR * 4) {  // four loads in flight per thread
            const float4 v0 = xv.at4(b, k), v1 = xv.at4(b, k + NTHR * 4), v2 = xv.at4(b, k + 2 * NTHR * 4),
                         v3 = xv.at4(b, k + 3 * NTHR * 4);
            *reinterpret_cast<float4 *>(xs + b * K + k) = v0;
            *reinterpret_cast<float4 *>(xs + b * K + k + NTHR * 4) = v1;
            *reinterpret_cast<float4 *>(xs + b * K + k + 2 * NTHR * 4) = v2;
            *reinterpret_cast<float4 *>(xs + b * K + k + 3 * NTHR * 4) = v3;
        }
        for (; k < K; k += NTHR * 4) *reinterpret_cast<float4 *>(xs + b * K + k) = xv.at4(b, k);
    }
    __syncthreads();
}

// Shared memory of a latency-GEMV op below the ring: xs, mean/rstd, acc.
__host__ __device__ __forceinline__ size_t fgemv_acc_off(int KB, int nb) { return (size_t)nb * KB * 256 * 4 + 16; }
__host__ __device__ __forceinline__ size_t fgemv_smem(int KB, int nb, int maxrt) {
    return fgemv_acc_off(KB, nb) + (size_t)maxrt * 2 * 16 * 4;
}

// One GEMV op (the body of k_gemv_tiled with clusters of one CTA): this CTA
// owns row tiles [t0, t1) whole, so every tile is finished here.
// Returns GEMV_OK when no ring wait ran out, plus GEMV_LATE when this warp
// still has to start the next GEMV's weight copies (after the op's outputs
// are out: the caller does it between the barrier's two phases).
constexpr int GEMV_OK = 1, GEMV_LATE = 2;
template <int QT, bool FF>
__device__ __forceinline__ int gemv_op_impl(uint8_t *smem, const DOp &op, Ring &r, StepCtl *ctl) {
    constexpr int NB = 2, UNIT = unit_bytes(QT);
    const TArgs &a = op.g;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int w0, w1, t0, t1;
    const bool mine = warp_units(a, blockIdx.x, wid, w0, w1, t0, t1);
    // the residual this warp's first tile adds to, loaded now (it is only
    // needed in the epilogue) so its latency hides behind the work below
    float pre = 0.0f, pbias = 0.0f;
    const bool has_pre = mine && (a.epi & LMC_EPI_ACCUM) && wid < t1 - t0;
    const bool has_pb = mine && a.bias && wid < t1 - t0;
    if (has_pre || has_pb) {
        const int row = (t0 + wid) * 16 + (lane & 15);
        if ((lane >> 4) < a.nb && row < a.M) {
            if (has_pre) pre = __ldcg(a.y + (size_t)(lane >> 4) * a.ldy + row);
            if (has_pb) pbias = __ldg(a.bias + row);
        }
    }
    const Smem<1, QT> L{a.KB, a.XL, a.maxrt, 0};
    float *acc = reinterpret_cast<float *>(smem + (FF ? fgemv_acc_off(a.KB, a.nb) : L.acc_off()));
    bool ok = true;
    if (mine) {
        for (int i = threadIdx.x; i < a.maxrt * NB * 16; i += NTHR) acc[i] = 0.0f;
        if (FF) load_x_f32(reinterpret_cast<float *>(smem), reinterpret_cast<float *>(smem + fgemv_acc_off(a.KB, a.nb) - 16), a);
        else build_x<1, QT, 0, true>(smem, L, a);
        __syncthreads();
        const float *inv = reinterpret_cast<const float *>(smem + L.sc_off()) + 8;
        const int XS = a.XL * XSTR, KB = a.KB, K = KB * 256;
        const uint8_t *xbl = smem + lane * XSTR;
        const uint32_t *xml = reinterpret_cast<const uint32_t *>(smem + L.xm_off()) + lane;
        const float *xsf = reinterpret_cast<const float *>(smem);
        const uint8_t *wbase = a.w + (size_t)t0 * KB * UNIT;
        Part<1> p;
        p.zero();
        FAcc fa;
        fa.zero();
        int cur = -1;
        int rt = w0 / KB, kb = w0 - rt * KB, s = r.s, i = w0;
        uint32_t parity = r.par;
        const int stages = r.stages, pf = a.pf;
        for (; i < w1; i++) {
            if (!mbar_wait(&r.bars[s], parity)) {
                ok = false;
                break;
            }
            r.inflight--;
            if (rt != cur) {
                if (cur >= 0) {
                    if (FF) fflush(fa, acc + cur * NB * 16, a.nb, lane);
                    else flush<1>(p, acc + cur * NB * 16, inv, a.nb, lane);
                }
                p.zero();
                fa.zero();
                cur = rt;
            }
            const uint8_t *u = r.slots + (size_t)s * SLOT;
            if (FF) {
                if (a.nb == 1) {
                    if (QT == 4) funit_q4k<1>(fa, u, xsf, K, kb * 256, lane);
                    else if (QT == 6) funit_q6k<1>(fa, u, xsf, K, kb * 256, lane);
                    else funit_q80<1>(fa, u, xsf, K, kb * 256, lane);
                } else {
                    if (QT == 4) funit_q4k<2>(fa, u, xsf, K, kb * 256, lane);
                    else if (QT == 6) funit_q6k<2>(fa, u, xsf, K, kb * 256, lane);
                    else funit_q80<2>(fa, u, xsf, K, kb * 256, lane);
                }
            } else {
                const uint8_t *xb = xbl + kb * XS;
                if (QT == 4) unit_q4k<1>(p, u, xb, XS, xml + kb * 32, lane);
                else if (QT == 6) unit_q6k<1>(p, u, xb, XS, xml + kb * 32, lane);
                else unit_q80<1>(p, u, xb, XS, lane);
            }
            __syncwarp();
            if (i + stages < w1) {
                refill(lane == 0, &r.bars[s], r.slots + (size_t)s * SLOT, wbase + (size_t)(i + stages) * UNIT, UNIT,
                       wbase + (size_t)(i + stages + pf) * UNIT, i + stages + pf < w1);
                r.inflight++;
            }
            if (++kb == KB) {
                kb = 0;
                rt++;
            }
            if (++s == stages) {
                s = 0;
                parity ^= 1u;
            }
        }
        r.s = s;
        r.par = parity;
        if (cur >= 0 && ok) {
            if (FF) fflush(fa, acc + cur * NB * 16, a.nb, lane);
            else flush<1>(p, acc + cur * NB * 16, inv, a.nb, lane);
        }
    }
    // this warp's slots are all consumed: start the next GEMV's weights - now
    // for a warp that had no units here, after the epilogue for the others
    // (issuing the copies is slow enough to delay the epilogue)
    const bool late_prefill = ok && op.next_gemv >= 0 && w1 > w0;
    if (!ok) {
        atomicExch(&ctl->abort, 1);
    } else if (op.next_gemv >= 0 && !late_prefill) {
        ring_prefill(r, op.ng, op.nqt, lane, wid);
    }
    if (!mine) return ok ? GEMV_OK : 0;
    __syncthreads();
    unsigned long long best = 0ull;
    double st[2] = {0.0, 0.0};
    if (a.epi & LMC_EPI_GLU_PAIRS) {  // y = silu(gate) * up per row of each (gate, up) tile pair
        for (int T = wid; T < (t1 - t0) >> 1; T += WARPS) {
            const int bb = lane >> 4, row = ((t0 >> 1) + T) * 16 + (lane & 15);
            if (bb < a.nb && 2 * row < a.M) {
                const float gv = acc[2 * T * NB * 16 + lane], uv = acc[(2 * T + 1) * NB * 16 + lane];
                a.y[(size_t)bb * a.ldy + row] = silu_short(gv) * uv;
            }
        }
        return (ok ? GEMV_OK : 0) | (late_prefill ? GEMV_LATE : 0);
    }
    for (int T = wid; T < t1 - t0; T += WARPS)
        step_epilogue_tile(a, (t0 + T) * 16, acc + T * NB * 16, lane, best, T == wid && has_pre ? &pre : nullptr,
                           T == wid && has_pb ? &pbias : nullptr, st);
    if (a.stats_out) {  // sums of this CTA's outputs for the next norm: fp32 in the half-warp of a batch row, fp64 across
#pragma unroll
        for (int q = 0; q < 2; q++) {
            float v = (float)st[q];
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if ((lane & 15) == 0 && (lane >> 4) < a.nb && v != 0.0f) atomicAdd(a.stats_out + 2 * (lane >> 4) + q, (double)v);
        }
    }
    if (a.keys) {  // greedy keys: half-warp maxima, then one atomic per CTA and batch row
        auto kbest = reinterpret_cast<unsigned long long(*)[2]>(smem);
        __syncthreads();  // the x fragments at offset 0 are dead
        unsigned long long k = best;
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
            k = o > k ? o : k;
        }
        if ((lane & 15) == 0) kbest[wid][lane >> 4] = k;
        __syncthreads();
        if ((int)threadIdx.x < a.nb) {
            unsigned long long k = 0ull;
            for (int w = 0; w < WARPS; w++) k = kbest[w][threadIdx.x] > k ? kbest[w][threadIdx.x] : k;
            if (k) atomicMax(a.keys + threadIdx.x, k);
        }
    }
    return (ok ? GEMV_OK : 0) | (late_prefill ? GEMV_LATE : 0);
}

// The attention body of the persistent step for at most two query heads per
// kv head.  Warp w takes positions t0 + w, t0 + w + 8, ...; lane l holds dims
// [DPL l, DPL l + DPL) of q, of the K and V rows and of the output, so a
// score is DPL FMAs per lane and a warp reduction, and a K or V row is one
// vector load per lane.  Each warp keeps an online softmax over its
// positions (running max, sum and accumulator), with the loads of a pass of
// PP positions issued before any is used; the eight warps' states are then
// merged in shared memory.  The new row (position pos) is made in registers
// by the warp that owns it - K rotated, rounded to the cache form - and
// stored to the cache from there.  One L2 round trip for q and the rows
// instead of the split body's five.  Same statistics and output format as
// split_body (so attn_merge_last merges either).
template <typename KV, int DH>
__device__ __forceinline__ void attn_short(const AttnArgs &a, float *sm, int kh, int b, int pos, int t0, int t1,
                                           float *wsb, size_t hstride, bool single) {
    constexpr int DPL = DH / 32, PP = DH == 64 ? 8 : 4;
    constexpr bool Q8 = KvT<KV>::Q8, F16 = sizeof(KV) == 2;
    const int G = a.H / a.Hkv, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, d0 = DPL * lane;
    const int RS = kv_rs<KV>(DH), n = t1 - t0;
    KV *kc = reinterpret_cast<KV *>(a.k_cache) + ((size_t)b * a.Hkv + kh) * a.S * RS;
    KV *vc = reinterpret_cast<KV *>(a.v_cache) + ((size_t)b * a.Hkv + kh) * a.S * RS;
    const float *rc = a.rope_cos ? a.rope_cos + (size_t)pos * (DH / 2) : nullptr;
    const float *rs = a.rope_sin ? a.rope_sin + (size_t)pos * (DH / 2) : nullptr;
    const float scale = 1.0f / sqrtf((float)DH);
    // q of the group's heads (rotated when RoPE applies)
    float q[2][DPL];
#pragma unroll
    for (int g = 0; g < 2; g++) {
        const float *qb = a.q + (size_t)b * a.ldq + ((size_t)kh * G + (g < G ? g : 0)) * DH + d0;
#pragma unroll
        for (int i = 0; i < DPL; i += 2) {
            float x0 = __ldcg(qb + i), x1 = __ldcg(qb + i + 1);
            if (rc) {
                const float c = rc[d0 / 2 + i / 2], sn = rs[d0 / 2 + i / 2];
                const float r0 = x0 * c - x1 * sn, r1 = x0 * sn + x1 * c;
                x0 = r0;
                x1 = r1;
            }
            q[g][i] = x0;
            q[g][i + 1] = x1;
        }
    }
    // the new row, made by the warp whose positions include it
    const int tp = pos - t0;
    const bool mine_new = tp >= 0 && tp < n && (tp & 7) == warp;
    float kn[DPL], vn[DPL], kns = 1.0f, vns = 1.0f;
    if (mine_new) {
        const float *kp = a.k_new + (size_t)b * a.ldkv + (size_t)kh * DH + d0;
        const float *vp = a.v_new + (size_t)b * a.ldkv + (size_t)kh * DH + d0;
#pragma unroll
        for (int i = 0; i < DPL; i += 2) {
            float x0 = __ldcg(kp + i), x1 = __ldcg(kp + i + 1);
            if (rc) {
                const float c = rc[d0 / 2 + i / 2], sn = rs[d0 / 2 + i / 2];
                const float r0 = x0 * c - x1 * sn, r1 = x0 * sn + x1 * c;
                x0 = r0;
                x1 = r1;
            }
            kn[i] = x0;
            kn[i + 1] = x1;
            vn[i] = __ldcg(vp + i);
            vn[i + 1] = __ldcg(vp + i + 1);
        }
        KV *kr = kc + (size_t)pos * RS, *vr = vc + (size_t)pos * RS;
        if constexpr (Q8) {  // as kv_q8_store_row: m = max|x| over the row, codes, scale
            float mk = 0.0f, mv = 0.0f;
#pragma unroll
            for (int i = 0; i < DPL; i++) {
                mk = fmaxf(mk, fabsf(kn[i]));
                mv = fmaxf(mv, fabsf(vn[i]));
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, off));
                mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, off));
            }
            const float ik = mk > 0.0f ? 127.0f / mk : 0.0f, iv = mv > 0.0f ? 127.0f / mv : 0.0f;
            int8_t *kq = reinterpret_cast<int8_t *>(kr), *vq = reinterpret_cast<int8_t *>(vr);
#pragma unroll
            for (int i = 0; i < DPL; i++) {
                const int ck = max(-127, min(127, __float2int_rn(__fmul_rn(kn[i], ik))));
                const int cv = max(-127, min(127, __float2int_rn(__fmul_rn(vn[i], iv))));
                kq[d0 + i] = (int8_t)ck;
                vq[d0 + i] = (int8_t)cv;
                kn[i] = (float)ck;  // K: codes (the score takes the row scale after the dot)
                vn[i] = (float)cv;
            }
            kns = mk / 127.0f;
            vns = mv / 127.0f;
            if (lane == 0) {
                *reinterpret_cast<float *>(kq + DH) = kns;
                *reinterpret_cast<float *>(vq + DH) = vns;
            }
#pragma unroll
            for (int i = 0; i < DPL; i++) vn[i] *= vns;
        } else {
#pragma unroll
            for (int i = 0; i < DPL; i++) {
                kr[d0 + i] = kv_cvt<KV>(kn[i]);
                vr[d0 + i] = kv_cvt<KV>(vn[i]);
                if (F16) {
                    kn[i] = __half2float(__float2half_rn(kn[i]));
                    vn[i] = __half2float(__float2half_rn(vn[i]));
                }
            }
        }
    }
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f}, acc[2][DPL];
#pragma unroll
    for (int g = 0; g < 2; g++)
#pragma unroll
        for (int i = 0; i < DPL; i++) acc[g][i] = 0.0f;
    for (int p0 = warp; p0 < n; p0 += 8 * PP) {
        float kr[PP][DPL], vr[PP][DPL], ks[PP], vs[PP];
#pragma unroll
        for (int j = 0; j < PP; j++) {  // every load of the pass in flight
            const int t = p0 + 8 * j;
            ks[j] = vs[j] = 1.0f;
#pragma unroll
            for (int i = 0; i < DPL; i++) kr[j][i] = vr[j][i] = 0.0f;
            if (t < n && t != tp) {
                const KV *kp = kc + (size_t)(t0 + t) * RS + d0, *vp = vc + (size_t)(t0 + t) * RS + d0;
#pragma unroll
                for (int i = 0; i < DPL; i++) {
                    kr[j][i] = kv_ld<KV>(kp + i);
                    vr[j][i] = kv_ld<KV>(vp + i);
                }
                if constexpr (Q8) {
                    ks[j] = kv_q8_scale(reinterpret_cast<const KvQ8 *>(kc + (size_t)(t0 + t) * RS), DH);
                    vs[j] = kv_q8_scale(reinterpret_cast<const KvQ8 *>(vc + (size_t)(t0 + t) * RS), DH);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < PP; j++) {
            const int t = p0 + 8 * j;
            if (t >= n) break;
            if (t == tp) {
#pragma unroll
                for (int i = 0; i < DPL; i++) {
                    kr[j][i] = kn[i];
                    vr[j][i] = vn[i];
                }
                ks[j] = kns;
            } else if (Q8) {
#pragma unroll
                for (int i = 0; i < DPL; i++) vr[j][i] *= vs[j];
            }
#pragma unroll
            for (int g = 0; g < 2; g++) {
                if (g >= G) break;
                float s = 0.0f;
#pragma unroll
                for (int i = 0; i < DPL; i++) s = fmaf(q[g][i], kr[j][i], s);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                s = (Q8 ? s * ks[j] : s) * scale;
                const float mn = fmaxf(m[g], s), c = expf(m[g] - mn), e = expf(s - mn);
                l[g] = l[g] * c + e;
#pragma unroll
                for (int i = 0; i < DPL; i++) acc[g][i] = fmaf(e, vr[j][i], acc[g][i] * c);
                m[g] = mn;
            }
        }
    }
    // merge the warps: [warp][g][DH + 2]
    float *st = sm;
#pragma unroll
    for (int g = 0; g < 2; g++) {
        if (g >= G) break;
        float *w = st + (warp * 2 + g) * (DH + 2);
#pragma unroll
        for (int i = 0; i < DPL; i++) w[d0 + i] = acc[g][i];
        if (lane == 0) {
            w[DH] = m[g];
            w[DH + 1] = l[g];
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * DH; idx += NTHR) {
        const int g = idx / DH, d = idx % DH;
        float M = -INFINITY;
        for (int w = 0; w < WARPS; w++) M = fmaxf(M, st[(w * 2 + g) * (DH + 2) + DH]);
        float L = 0.0f, o = 0.0f;
        for (int w = 0; w < WARPS; w++) {
            const float *x = st + (w * 2 + g) * (DH + 2);
            if (x[DH + 1] == 0.0f) continue;  // a warp with no positions
            const float f = expf(x[DH] - M);
            L += x[DH + 1] * f;
            o += x[d] * f;
        }
        if (single) {
            a.out[(size_t)b * a.ldo + ((size_t)kh * G + g) * DH + d] = o / L;
        } else {
            wsb[g * hstride + d] = o;
            if (d == 0) {
                wsb[g * hstride + DH] = M;
                wsb[g * hstride + DH + 1] = L;
            }
        }
    }
}

// Attention work items (split, kv head, sequence), dealt round-robin to the
// CTAs; the last split of each (sequence, kv head) to finish merges them.
// The plan's splits are sized for the longest context; at the current
// position they are coarsened (doubled) up to ATT_ONE_SPLIT positions, so a
// context that short is one split per head (no merge, which costs a
// fence, an arrival atomic and a read-back of the partials), and a longer
// one is split into pieces of at least that many positions.
constexpr int ATT_ONE_SPLIT = 256;  // one scores pass of 8 warps x 32 lanes
template <typename KV, int DH>
__device__ __forceinline__ void attn_op(uint8_t *smem, const AttnArgs &a, int items, int *sh_last) {
    const int G = a.H / a.Hkv, Dh = a.Dh;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int sp = it % a.nsplit, r2 = it / a.nsplit, kh = r2 % a.Hkv, b = r2 / a.Hkv;
        const int pos = __ldcg(a.pos + b);
        if (pos < 0 || pos >= a.S) continue;  // the host validates positions
        int CH = a.CH;
        while (CH < ATT_ONE_SPLIT && CH <= pos) CH *= 2;
        const int t0 = sp * CH, t1 = min(t0 + CH, pos + 1);
        if (t0 > pos) continue;
        const bool single = pos < CH;
        float *wsb = a.ws + (((size_t)b * a.H + (size_t)kh * G) * a.nsplit + sp) * (Dh + 2);
        const size_t hstride = (size_t)a.nsplit * (Dh + 2);
        // the short body for head size 64 with fp32 rows (LMc's cache); with
        // the other forms as well the kernel would exceed its 128 registers
        if (DH == 64 && sizeof(KV) == 4 && G <= 2 && t1 - t0 <= ATT_ONE_SPLIT)
            attn_short<KV, DH>(a, reinterpret_cast<float *>(smem), kh, b, pos, t0, t1, wsb, hstride, single);
        else
            split_body<KV, DH, NTHR, 128>(a, reinterpret_cast<float *>(smem), sp, kh, b, pos, t0, t1, wsb, hstride,
                                          CH, single);
        if (!single) attn_merge_last<NTHR>(a, wsb, hstride, kh, b, pos, sh_last, CH);
        __syncthreads();  // shared memory is reused by the next item
    }
}

template <int T>
__device__ __forceinline__ void embed_row(const EmbedArgs &e, int b, double (&st)[2]) {
    using F = lmcq::Fmt<T>;
    const int tok = __ldcg(e.tok + b), pos = e.wpe ? __ldcg(e.pos + b) : 0;
    if (tok < 0 || tok >= e.V || pos < 0 || pos >= e.S) return;  // the host validates tokens and positions
    const size_t r0 = (size_t)tok * e.D, r1 = r0 + e.D;
    for (size_t g = (r0 >> 3) + threadIdx.x; g < ((r1 + 7) >> 3); g += NTHR) {
        const size_t el = g << 3;
        float w[8];
        lmcq::decode8<T>(e.wte + (el / F::BE) * F::BB, (int)(el % F::BE), w);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const long long k = (long long)(el + i) - (long long)r0;
            if (k >= 0 && k < e.D) {
                float v = w[i];
                if (e.wpe) v = v + e.wpe[(size_t)pos * e.D + k];
                e.out[(size_t)b * e.D + k] = v;
                st[0] += (double)v;
                st[1] += (double)v * (double)v;
            }
        }
    }
}

// One CTA per sequence row; the row's fp64 sums (for the first norm) are
// stored, not added, so they need no zeroing.
__device__ __forceinline__ void embed_op(const EmbedArgs &e, int nb, double *red) {
    for (int b = blockIdx.x; b < nb; b += gridDim.x) {
        double st[2] = {0.0, 0.0};
        switch (e.type) {
        case LMC_TYPE_Q4_K: embed_row<LMC_TYPE_Q4_K>(e, b, st); break;
        case LMC_TYPE_Q6_K: embed_row<LMC_TYPE_Q6_K>(e, b, st); break;
        case LMC_TYPE_Q8_0: embed_row<LMC_TYPE_Q8_0>(e, b, st); break;
        case LMC_TYPE_F16: embed_row<LMC_TYPE_F16>(e, b, st); break;
        default: embed_row<LMC_TYPE_F32>(e, b, st); break;
        }
        if (!e.stats_out) continue;
#pragma unroll
        for (int q = 0; q < 2; q++) {
            double v = st[q];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if ((threadIdx.x & 31) == 0) red[2 * (threadIdx.x >> 5) + q] = v;
        }
        __syncthreads();
        if (threadIdx.x < 2) {
            double t = 0.0;
            for (int w = 0; w < WARPS; w++) t += red[2 * w + threadIdx.x];
            e.stats_out[2 * b + threadIdx.x] = t;
        }
        __syncthreads();
    }
}

// Greedy pick of each sequence from its key (reset for the next step); with
// `generate`, the bookkeeping of k_advance (ops.cu): the next token is the
// next prompt token while the prompt lasts, then the pick, which is recorded.
__device__ __forceinline__ void advance_op(const AdvArgs &v, int nb) {
    if (blockIdx.x != 0) return;
    const int step = v.generate ? __ldcg(v.step) : 0;
    for (int b = threadIdx.x; b < nb; b += NTHR) {
        const int nx = v.from_next ? __ldcg(v.next + b) : lmc_key_index(__ldcg(v.keys + b));
        v.keys[b] = 0ull;
        v.next[b] = nx;
        if (v.next_host) v.next_host[b] = nx;
        if (!v.generate) continue;
        if (step + 1 < v.n_prompt) {
            v.tok[b] = v.prompt[(size_t)b * v.n_prompt + step + 1];
        } else {
            const int k = step + 1 - v.n_prompt;
            v.tok[b] = nx;
            if (k < v.n_new) v.ids[(size_t)b * v.n_new + k] = nx;
        }
        v.pos[b] = step + 1;
    }
    __syncthreads();
    if (v.generate && threadIdx.x == 0) *v.step = step + 1;
}

// One top-p draw per sequence (CTA b draws row b), only in steps whose pick
// is a generated token, as k_sample (sample.cu).
__device__ __forceinline__ void sample_op(uint8_t *smem, const SampArgs &a, int nb) {
    if (a.step && __ldcg(a.step) + 1 < a.n_prompt) return;
    for (int b = blockIdx.x; b < nb; b += gridDim.x)
        sample_row<NTHR>(a.logits + (size_t)b * a.V, a.V, a.temperature, a.top_p, a.rng + b, a.next + b,
                         *reinterpret_cast<SampleSmem *>(smem));
}

__global__ void __launch_bounds__(NTHR, 2) k_step(StepParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(16) DOp ops[2];  // op i in ops[i & 1]; op i + 1 is copied in during barrier i
    __shared__ int sh_ok, sh_last;
    __shared__ unsigned sh_base[BAR_GROUPS];
    __shared__ double sh_red[2 * WARPS];
    StepCtl *ctl = P.ctl;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (threadIdx.x == 0) sh_ok = *(volatile int *)&ctl->abort == 0;  // an earlier launch gave up: run nothing
    if (threadIdx.x < BAR_GROUPS) sh_base[threadIdx.x] = *(volatile unsigned *)&ctl->base[threadIdx.x];
    {
        const int4 *src = reinterpret_cast<const int4 *>(P.ops);
        int4 *dst = reinterpret_cast<int4 *>(&ops[0]);
        for (int w = threadIdx.x; w < (int)(sizeof(DOp) / 16); w += NTHR) dst[w] = __ldg(src + w);
    }
    if (threadIdx.x == 0 && (int)blockIdx.x < P.imm_n) {  // (no runtime index into the parameter arrays)
        P.tok_dst[blockIdx.x] = blockIdx.x ? P.imm_tok[1] : P.imm_tok[0];
        P.pos_dst[blockIdx.x] = blockIdx.x ? P.imm_pos[1] : P.imm_pos[0];
    }
    __syncthreads();
    if (!sh_ok) return;
    Ring r;
    r.stages = P.stages;
    r.slots = smem + P.ring_off + (size_t)wid * P.stages * SLOT;
    r.bars = reinterpret_cast<uint64_t *>(smem + P.ring_off + (size_t)WARPS * P.stages * SLOT) + wid * P.stages;
    r.s = 0;
    r.par = 0;
    r.inflight = 0;
    if (lane == 0) {
        for (int s = 0; s < P.stages; s++) mbar_init(&r.bars[s]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (threadIdx.x == 64)
        for (int k = blockIdx.x; k < P.pf_n; k += gridDim.x) prefetch_l2(P.pf[k].p, P.pf[k].bytes);
    if (P.first_gemv >= 0) ring_prefill(r, P.ops[P.first_gemv].g, P.ops[P.first_gemv].qt, lane, wid);
    unsigned passed = 0;
    bool alive = true;
    for (int i = 0; i < P.nops && alive; i++) {
        const DOp &op = ops[i & 1];
        int gres = 0;
        switch (op.kind) {
        case LMC_OP_EMBED: embed_op(op.e, op.nb, sh_red); break;
        case LMC_OP_GEMV:
            if (op.ff) {
                if (op.qt == 4) gres = gemv_op_impl<4, true>(smem, op, r, ctl);
                else if (op.qt == 6) gres = gemv_op_impl<6, true>(smem, op, r, ctl);
                else gres = gemv_op_impl<8, true>(smem, op, r, ctl);
            } else {
                if (op.qt == 4) gres = gemv_op_impl<4, false>(smem, op, r, ctl);
                else if (op.qt == 6) gres = gemv_op_impl<6, false>(smem, op, r, ctl);
                else gres = gemv_op_impl<8, false>(smem, op, r, ctl);
            }
            alive = (gres & GEMV_OK) != 0;
            break;
        case LMC_OP_ATTN:
            if (op.kv == LMC_KV_F32) {
                if (op.dh == 64) attn_op<float, 64>(smem, op.at, op.items, &sh_last);
                else attn_op<float, 128>(smem, op.at, op.items, &sh_last);
            } else if (op.kv == LMC_KV_Q8) {
                if (op.dh == 64) attn_op<KvQ8, 64>(smem, op.at, op.items, &sh_last);
                else attn_op<KvQ8, 128>(smem, op.at, op.items, &sh_last);
            } else {
                if (op.dh == 64) attn_op<__half, 64>(smem, op.at, op.items, &sh_last);
                else attn_op<__half, 128>(smem, op.at, op.items, &sh_last);
            }
            break;
        case LMC_OP_SAMPLE: sample_op(smem, op.sm, op.nb); break;
        default: advance_op(op.v, op.nb); break;
        }
        const DOp *nsrc = i + 1 < P.nops ? P.ops + i + 1 : nullptr;
        if (op.sync) {
            // a ring wait that ran out in any warp of any CTA aborts the step
            // here (grid_wait polls the flag)
            passed++;
            grid_arrive(ctl);
            // in the barrier's shadow: the next GEMV's first weight copies for
            // warps that had units here, and the K/V rows of a coming attention
            if (gres & GEMV_LATE) ring_prefill(r, op.ng, op.nqt, lane, wid);
            if (op.kind == LMC_OP_GEMV && op.kpf) kv_prefetch(op.kp);
            alive = grid_wait(ctl, sh_base, passed, i, &sh_ok, nsrc, &ops[(i + 1) & 1]) && alive;
        } else {
            __syncthreads();
            if (nsrc) {
                const int4 *src = reinterpret_cast<const int4 *>(nsrc);
                int4 *dst = reinterpret_cast<int4 *>(&ops[(i + 1) & 1]);
                for (int w = threadIdx.x; w < (int)(sizeof(DOp) / 16); w += NTHR) dst[w] = __ldg(src + w);
            }
            __syncthreads();
        }
    }
    if (alive && blockIdx.x == 0) {
        if (threadIdx.x < BAR_GROUPS) ctl->base[threadIdx.x] = sh_base[threadIdx.x] + passed * group_size(threadIdx.x);
        // every norm has read its statistics (before the last barrier): zero
        // the slots for the next launch
        for (int k = threadIdx.x; k < P.stats_n; k += NTHR) P.stats[k] = 0.0;
    }
    // after an abort: wait (bounded) for this warp's copies still in flight
    if (lane == 0 && r.inflight > 0) {
        int s = r.s;
        uint32_t par = r.par;
        for (int k = 0; k < r.inflight; k++) {
            (void)mbar_wait(&r.bars[s], par);
            if (++s == r.stages) {
                s = 0;
                par ^= 1u;
            }
        }
    }
}

// Failure-path self-test of the grid barrier: the counters' base is set so
// that the first barrier can never complete (a count nothing reaches); every
// CTA gives up after the wait limit, raises the abort flag and returns.
__global__ void k_barrier_selftest(StepCtl *ctl, int *left) {
    __shared__ int sh_ok;
    __shared__ unsigned base[BAR_GROUPS];
    if (threadIdx.x < BAR_GROUPS) base[threadIdx.x] = 0x40000000u;
    __syncthreads();
    const bool ok = grid_sync(ctl, base, 1, 0, &sh_ok, nullptr, nullptr);
    if (threadIdx.x == 0 && !ok) atomicAdd(left, 1);
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct lmc_step_prog {
    DOp *d_ops;
    int nops, first_gemv, grid, stages, ring_off;
    size_t smem;
    StepCtl *ctl;
    double *stats;
    int stats_n;
    PfRange *pf;
    int pf_n;
};
constexpr int STATS_STRIDE = 4;  // doubles per slot: {sum, sum of squares} x 2 batch rows

static std::vector<lmc_step_prog *> g_progs;  // live programs, for lmc_step_status
static std::mutex g_progs_mu;

static int qt_of_type(uint32_t t) { return t == LMC_TYPE_Q4_K ? 4 : t == LMC_TYPE_Q6_K ? 6 : 8; }

static size_t gemv_smem(int qt, int KB, int XL, int maxrt) {
    if (qt == 4) return Smem<1, 4>{KB, XL, maxrt, 0}.ring_off();
    if (qt == 6) return Smem<1, 6>{KB, XL, maxrt, 0}.ring_off();
    return Smem<1, 8>{KB, XL, maxrt, 0}.ring_off();
}

// Fills the GEMV fields of `d` for a grid of `grid` CTAs; returns the shared
// memory below the ring that the op needs, or 0 when it cannot run here.
static size_t plan_gemv(const lmc_step_op *o, int grid, int stages, DOp *d) {
    const lmc_qtensor *t = o->w;
    if (!t || !t->tiled || o->batch < 1 || o->batch > 2) return 0;
    const lmc_gemv_extra *ex = &o->ex;
    if (((uintptr_t)o->x & 15) || (o->ldx & 3) || (ex->x2 && ((uintptr_t)ex->x2 & 15)) ||
        (ex->w && ((uintptr_t)ex->w & 15)) || (ex->b && ((uintptr_t)ex->b & 15)))
        return 0;
    TArgs a = {};
    a.w = (const uint8_t *)t->tiled;
    a.x = o->x;
    a.bias = o->bias;
    a.y = o->y;
    a.M = t->rows;
    a.KB = t->cols / 256;
    a.RT = t->tiled_rows / 16;
    a.ldx = o->ldx;
    a.ldy = o->ldy;
    a.nb = o->batch;
    a.epi = o->epi;
    a.pro = ex->pro;
    a.pw = ex->w;
    a.pb = ex->b;
    a.x2 = ex->x2;
    a.eps = ex->eps;
    a.keys = ex->keys;
    a.key_base = ex->key_base;
    a.XL = 12 * o->batch;
    a.CL = 1;
    if (a.epi & LMC_EPI_GLU_PAIRS) {
        if ((a.RT & 1) || t->rows != t->tiled_rows || ex->keys || o->bias) return 0;
        a.NC = std::min(grid, a.RT / 2);
        a.maxrt = 2 * ((a.RT / 2 + a.NC - 1) / a.NC) + 1;
    } else {
        a.NC = std::min(grid, a.RT);
        a.maxrt = (a.RT + a.NC - 1) / a.NC + 1;
    }
    a.stages = stages;
    const int qt = qt_of_type(t->type);
    // no L2 prefetch of the units beyond the ring: with the ring prefill in
    // the barrier's shadow it only queued HBM traffic ahead of the ops'
    // demand loads (GPT-2 Small 0.396 -> 0.393 ms, 8B shape 3.33 -> 3.24 ms
    // per step without a 40 MB window)
    a.pf = 0;
    d->g = a;
    d->qt = qt;
    // the latency form when a warp gets few units, x fits in shared memory as
    // fp32, and a norm prologue has its statistics from the op that wrote x
    // (LMC_STEP_FF=0: the tensor-core form everywhere; same results to fp32
    // rounding)
    const char *env = getenv("LMC_STEP_FF");
    const long long per_warp = ((long long)(a.maxrt - 1) * a.KB + WARPS - 1) / WARPS;
    const bool norm = a.pro == LMC_PRO_LAYERNORM || a.pro == LMC_PRO_RMSNORM;
    d->ff = !(env && env[0] == '0') && per_warp <= 8 && (size_t)o->batch * a.KB * 1024 <= 64 * 1024 &&
            (!norm || o->stats_in);
    return d->ff ? fgemv_smem(a.KB, o->batch, a.maxrt) : gemv_smem(qt, a.KB, a.XL, a.maxrt);
}

static size_t plan_attn(const lmc_step_op *o, DOp *d) {
    if (!o->out || !o->q || !o->k_new || !o->v_new || !o->k_cache || !o->v_cache || !o->pos || !o->cnt) return 0;
    if (o->batch <= 0 || o->H <= 0 || o->Hkv <= 0 || o->H % o->Hkv || (o->Dh != 64 && o->Dh != 128) || o->S <= 0)
        return 0;
    if (o->kv_dtype != LMC_KV_F32 && o->kv_dtype != LMC_KV_F16 && o->kv_dtype != LMC_KV_Q8) return 0;
    AttnArgs a = {};
    a.out = o->out;
    a.q = o->q;
    a.k_new = o->k_new;
    a.v_new = o->v_new;
    a.k_cache = o->k_cache;
    a.v_cache = o->v_cache;
    a.pos = o->pos;
    a.H = o->H;
    a.Hkv = o->Hkv;
    a.Dh = o->Dh;
    a.S = o->S;
    a.ldo = o->ldo;
    a.ldq = o->ldq;
    a.ldkv = o->ldkv;
    a.rope_cos = o->rope_cos;
    a.rope_sin = o->rope_sin;
    a.cnt = o->cnt;
    a.seq = NULL;
    a.append = 1;
    lmc_attn_plan(o->S, o->batch * o->H, 1, &a.CH, &a.nsplit);
    const size_t need = a.nsplit > 1 ? (size_t)o->batch * o->H * a.nsplit * (o->Dh + 2) * sizeof(float) : 0;
    if (need > o->ws_bytes || (need && !o->ws)) return 0;
    a.ws = (float *)o->ws;
    d->at = a;
    d->kv = o->kv_dtype;
    d->dh = o->Dh;
    d->items = a.nsplit * o->Hkv * o->batch;
    const int G = o->H / o->Hkv;
    // scores of up to max(CH, ATT_ONE_SPLIT) positions per split (attn_op coarsens the plan)
    return (size_t)(G * o->Dh + G * std::max(a.CH, ATT_ONE_SPLIT) + 2 * G + WARPS * ATT_GROUP * o->Dh) * sizeof(float);
}

extern "C" int lmc_step_prog_build(const lmc_step_op *ops, int n, lmc_step_prog **out) {
    if (!ops || n <= 0 || !out) return lmc_set_error(LMC_ERR_INVALID, "step_prog: args");
    *out = NULL;
    int dev = 0;
    LMC_CUDA_TRY(cudaGetDevice(&dev));
    int coop = 0;
    LMC_CUDA_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
    if (!coop) return lmc_set_error(LMC_ERR_UNSUPPORTED, "step_prog: no cooperative launch");
    const int sms = lmc_sm_count();
    std::vector<DOp> d((size_t)n);
    // two CTAs per SM when the shared memory allows, else one; the deepest ring that fits
    const int shapes[5][2] = {{2, 3}, {2, 2}, {1, 4}, {1, 3}, {1, 2}};
    int grid = 0, stages = 0;
    size_t below = 0, smem = 0;
    for (int si = 0; si < 5 && !grid; si++) {
        const int cps = shapes[si][0], st = shapes[si][1], g = sms * cps;
        size_t need = 512;  // greedy-key scratch at offset 0
        bool ok = true;
        for (int i = 0; i < n && ok; i++) {
            memset(&d[i], 0, sizeof(DOp));
            d[i].kind = ops[i].kind;
            d[i].nb = ops[i].batch;
            d[i].next_gemv = -1;
            size_t s = 1;
            switch (ops[i].kind) {
            case LMC_OP_GEMV: s = plan_gemv(&ops[i], g, st, &d[i]); break;
            case LMC_OP_ATTN: s = plan_attn(&ops[i], &d[i]); break;
            case LMC_OP_EMBED: {
                const uint32_t ty = ops[i].wte_type;
                if (ty != LMC_TYPE_Q4_K && ty != LMC_TYPE_Q6_K && ty != LMC_TYPE_Q8_0 && ty != LMC_TYPE_F16 &&
                    ty != LMC_TYPE_F32)
                    s = 0;
                d[i].e = EmbedArgs{(const uint8_t *)ops[i].wte, ops[i].wpe, ops[i].tok, ops[i].pos, ops[i].D,
                                   ops[i].V, ops[i].S, (int)ty, ops[i].y, nullptr};
                break;
            }
            case LMC_OP_SAMPLE:
                d[i].sm = SampArgs{ops[i].y, ops[i].V, ops[i].temperature, ops[i].top_p, ops[i].rng, ops[i].next,
                                   ops[i].step, ops[i].n_prompt};
                if (!ops[i].y || !ops[i].rng || !ops[i].next || ops[i].V <= 0) s = 0;
                else s = sizeof(SampleSmem);
                break;
            case LMC_OP_KEYS:
            case LMC_OP_ADVANCE:
                d[i].v = AdvArgs{ops[i].keys, ops[i].next, ops[i].tok, ops[i].pos, ops[i].step, ops[i].ids,
                                 ops[i].next_host, ops[i].prompt, ops[i].n_prompt, ops[i].n_new,
                                 ops[i].kind == LMC_OP_ADVANCE, ops[i].from_next};
                if (!ops[i].keys || !ops[i].next ||
                    (ops[i].kind == LMC_OP_ADVANCE && (!ops[i].tok || !ops[i].pos || !ops[i].step || !ops[i].prompt ||
                                                       !ops[i].ids)))
                    s = 0;
                break;
            default: s = 0;
            }
            if (!s) {
                ok = false;
                break;
            }
            need = std::max(need, s);
            // every op but a trailing bookkeeping op is followed by a barrier
            d[i].sync = !(i == n - 1 && (ops[i].kind == LMC_OP_KEYS || ops[i].kind == LMC_OP_ADVANCE));
        }
        if (!ok) return lmc_set_error(LMC_ERR_UNSUPPORTED, "step_prog: an op has no persistent form");
        need = (need + 127) / 128 * 128;
        const size_t tot = need + (size_t)WARPS * st * SLOT + (size_t)WARPS * st * 8;
        if (tot > (size_t)(cps == 2 ? 112 * 1024 : 220 * 1024)) continue;
        if (cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tot) != cudaSuccess) {
            (void)cudaGetLastError();
            continue;
        }
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step, NTHR, tot) != cudaSuccess) {
            (void)cudaGetLastError();
            continue;
        }
        if (per_sm < cps) continue;
        grid = g;
        stages = st;
        below = need;
        smem = tot;
    }
    if (!grid) return lmc_set_error(LMC_ERR_UNSUPPORTED, "step_prog: does not fit one grid");
    int first = -1;
    for (int i = n - 1, nxt = -1; i >= 0; i--) {
        d[i].next_gemv = nxt;
        if (nxt >= 0) {
            d[i].ng = d[nxt].g;
            d[i].nqt = d[nxt].qt;
        }
        if (d[i].kind == LMC_OP_GEMV) nxt = i;
        first = nxt;
    }
    // the K/V rows an attention op reads are asked of L2 at the end of the
    // GEMV two ops before it (one op before, when that is the first GEMV), so
    // they arrive while other work runs
    for (int i = 1; i < n; i++)
        if (d[i].kind == LMC_OP_ATTN) {
            const int j = i >= 2 && d[i - 2].kind == LMC_OP_GEMV ? i - 2 : d[i - 1].kind == LMC_OP_GEMV ? i - 1 : -1;
            if (j < 0) continue;
            const AttnArgs &at = d[i].at;
            d[j].kpf = 1;
            d[j].kp = KvPf{(const uint8_t *)at.k_cache, (const uint8_t *)at.v_cache, at.pos, at.Hkv, at.S,
                           (int)LMC_KV_ROW_BYTES(d[i].kv, at.Dh), d[i].nb};
        }
    int slots = 0;
    for (int i = 0; i < n; i++) slots = std::max(slots, std::max(ops[i].stats_in, ops[i].stats_out));
    lmc_step_prog *p = (lmc_step_prog *)calloc(1, sizeof(lmc_step_prog));
    if (!p) return lmc_set_error(LMC_ERR_OOM, "step_prog: host");
    p->nops = n;
    p->first_gemv = first;
    p->grid = grid;
    p->stages = stages;
    p->ring_off = (int)below;
    p->smem = smem;
    p->stats_n = slots * STATS_STRIDE;
    cudaError_t e = cudaMalloc((void **)&p->d_ops, sizeof(DOp) * n);
    if (e == cudaSuccess) e = cudaMalloc((void **)&p->ctl, sizeof(StepCtl));
    if (e == cudaSuccess && slots) e = cudaMalloc((void **)&p->stats, sizeof(double) * p->stats_n);
    if (e == cudaSuccess && slots) e = cudaMemset(p->stats, 0, sizeof(double) * p->stats_n);
    if (e == cudaSuccess && slots)
        for (int i = 0; i < n; i++) {
            double *in = ops[i].stats_in ? p->stats + (size_t)(ops[i].stats_in - 1) * STATS_STRIDE : nullptr;
            double *out = ops[i].stats_out ? p->stats + (size_t)(ops[i].stats_out - 1) * STATS_STRIDE : nullptr;
            if (d[i].kind == LMC_OP_GEMV) {
                d[i].g.stats = in;
                d[i].g.stats_out = out;
            } else if (d[i].kind == LMC_OP_EMBED) {
                d[i].e.stats_out = out;
            }
        }
    // the copies of the next GEMV's arguments pick up its statistics pointers
    for (int i = 0; i < n; i++)
        if (d[i].next_gemv >= 0) d[i].ng = d[d[i].next_gemv].g;
    if (e == cudaSuccess) e = cudaMemcpy(p->d_ops, d.data(), sizeof(DOp) * n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(p->ctl, 0, sizeof(StepCtl));
    // the small vectors of every GEMV (norm weights and biases), asked of L2
    // when the step starts
    std::vector<PfRange> pf;
    auto add_pf = [&pf](const void *v, size_t bytes) {
        if (!v || !bytes) return;
        const uintptr_t a0 = (uintptr_t)v & ~(uintptr_t)15, a1 = ((uintptr_t)v + bytes + 15) & ~(uintptr_t)15;
        pf.push_back(PfRange{(const void *)a0, (unsigned)(a1 - a0)});
    };
    for (int i = 0; i < n; i++)
        if (d[i].kind == LMC_OP_GEMV) {
            const TArgs &g = d[i].g;
            const size_t K = (size_t)g.KB * 256;
            add_pf(g.bias, (size_t)g.M * sizeof(float));
            if (g.pro == LMC_PRO_LAYERNORM || g.pro == LMC_PRO_RMSNORM) add_pf(g.pw, K * sizeof(float));
            if (g.pro == LMC_PRO_LAYERNORM) add_pf(g.pb, K * sizeof(float));
        }
    if (e == cudaSuccess && !pf.empty()) {
        e = cudaMalloc((void **)&p->pf, sizeof(PfRange) * pf.size());
        if (e == cudaSuccess) e = cudaMemcpy(p->pf, pf.data(), sizeof(PfRange) * pf.size(), cudaMemcpyHostToDevice);
        p->pf_n = (int)pf.size();
    }
    if (e != cudaSuccess) {
        lmc_step_prog_free(p);
        return lmc_set_error(LMC_ERR_CUDA, "step_prog: %s", cudaGetErrorString(e));
    }
    {
        std::lock_guard<std::mutex> lock(g_progs_mu);
        g_progs.push_back(p);
    }
    *out = p;
    return LMC_OK;
}

static int step_launch(const lmc_step_prog *p, cudaStream_t s, const int *h_tok, const int *h_pos, int nb,
                       int *d_tok, int *d_pos);
extern "C" int lmc_step_prog_launch(const lmc_step_prog *p, cudaStream_t s) {
    return step_launch(p, s, NULL, NULL, 0, NULL, NULL);
}
extern "C" int lmc_step_prog_launch_imm(const lmc_step_prog *p, cudaStream_t s, const int *h_tok, const int *h_pos,
                                        int nb, int *d_tok, int *d_pos) {
    if (!h_tok || !h_pos || !d_tok || !d_pos || nb < 1 || nb > 2)
        return lmc_set_error(LMC_ERR_INVALID, "step_prog_launch_imm: args");
    return step_launch(p, s, h_tok, h_pos, nb, d_tok, d_pos);
}
static int step_launch(const lmc_step_prog *p, cudaStream_t s, const int *h_tok, const int *h_pos, int nb,
                       int *d_tok, int *d_pos) {
    if (!p) return lmc_set_error(LMC_ERR_INVALID, "step_prog_launch: null");
    StepParams P;
    P.imm_n = nb;
    for (int b = 0; b < 2; b++) {
        P.imm_tok[b] = b < nb ? h_tok[b] : 0;
        P.imm_pos[b] = b < nb ? h_pos[b] : 0;
    }
    P.tok_dst = d_tok;
    P.pos_dst = d_pos;
    P.ops = p->d_ops;
    P.nops = p->nops;
    P.first_gemv = p->first_gemv;
    P.ring_off = p->ring_off;
    P.stages = p->stages;
    P.ctl = p->ctl;
    P.stats = p->stats;
    P.stats_n = p->stats_n;
    P.pf = p->pf;
    P.pf_n = p->pf_n;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(NTHR);
    cfg.dynamicSmemBytes = p->smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    void *args[1] = {&P};
    cudaError_t e = cudaLaunchKernelExC(&cfg, (const void *)k_step, args);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "persistent step launch: %s", cudaGetErrorString(e));
    return LMC_OK;
}

extern "C" void lmc_step_prog_free(lmc_step_prog *p) {
    if (!p) return;
    std::lock_guard<std::mutex> lock(g_progs_mu);
    for (size_t i = 0; i < g_progs.size(); i++)
        if (g_progs[i] == p) {
            g_progs.erase(g_progs.begin() + (long)i);
            break;
        }
    if (p->d_ops) cudaFree(p->d_ops);
    if (p->ctl) cudaFree(p->ctl);
    if (p->stats) cudaFree(p->stats);
    if (p->pf) cudaFree(p->pf);
    free(p);
}

extern "C" int lmc_step_status(void) {
    int rc = LMC_OK;
    int tiled = 0;
    if (cudaMemcpyFromSymbol(&tiled, g_tiled_timeout, sizeof(int)) != cudaSuccess)
        return lmc_set_error(LMC_ERR_CUDA, "step_status: read flag");
    if (tiled) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_tiled_timeout, &zero, sizeof(int));
        rc = lmc_set_error(LMC_ERR_TIMEOUT, "persistent step: a weight copy did not complete in time");
    }
    std::lock_guard<std::mutex> lock(g_progs_mu);
    for (lmc_step_prog *p : g_progs) {
        StepCtl c;
        if (cudaMemcpy(&c, p->ctl, sizeof c, cudaMemcpyDeviceToHost) != cudaSuccess)
            return lmc_set_error(LMC_ERR_CUDA, "step_status: read barrier state");
        if (c.abort) {  // the launch left its barrier counters and statistics mid-way
            cudaMemset(p->ctl, 0, sizeof(StepCtl));
            if (p->stats) cudaMemset(p->stats, 0, sizeof(double) * p->stats_n);
            rc = lmc_set_error(LMC_ERR_TIMEOUT, "persistent step: a grid barrier wait ran out (op %d)", c.where - 1);
        }
    }
    return rc;
}

extern "C" int lmc_step_set_wait_limit(long long ns) {
    const long long v = ns > 0 ? ns : 1000000000ll;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_step_wait_ns, &v, sizeof v));
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_wait_ns, &v, sizeof v));
    return LMC_OK;
}

extern "C" int lmc_step_barrier_selftest(int *d_left, cudaStream_t s) {
    StepCtl *ctl = NULL;
    LMC_CUDA_TRY(cudaMalloc((void **)&ctl, sizeof(StepCtl)));
    cudaError_t e = cudaMemset(ctl, 0, sizeof(StepCtl));
    if (e == cudaSuccess) {
        void *args[2] = {&ctl, &d_left};
        e = cudaLaunchCooperativeKernel((const void *)k_barrier_selftest, dim3(2), dim3(NTHR), args, 0, s);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    StepCtl c;
    if (e == cudaSuccess) e = cudaMemcpy(&c, ctl, sizeof c, cudaMemcpyDeviceToHost);
    cudaFree(ctl);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "barrier self-test: %s", cudaGetErrorString(e));
    return c.abort ? lmc_set_error(LMC_ERR_TIMEOUT, "grid barrier wait ran out (self-test)") : LMC_OK;
}
