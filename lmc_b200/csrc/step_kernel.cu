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
};
struct AdvArgs {
    unsigned long long *keys;
    int *next, *tok, *pos, *step, *ids;
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
    int kv, dh;       // ATTN: 0 fp32 / 1 fp16 cache; head size 64 / 128
    int items;        // ATTN: splits x kv heads x batch
    TArgs g;
    AttnArgs at;
    EmbedArgs e;
    AdvArgs v;
    SampArgs sm;
};
struct StepCtl {
    unsigned count;  // barrier arrivals, never reset between launches
    unsigned base;   // count at the start of the next launch
    int abort;       // set when a wait ran out: every CTA leaves
    int where;       // op index + 1 of the wait that ran out
};
struct StepParams {
    const DOp *ops;
    int nops, first_gemv, ring_off, stages;
    StepCtl *ctl;
};

__device__ long long g_step_wait_ns = 1000000000ll;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier number `target` / gridDim.x: thread 0 of each CTA adds its
// arrival (after a fence, so the CTA's writes are visible) and polls until all
// arrived, the abort flag is set, or the wait limit passes (then it sets the
// flag).  Returns false when the CTA must leave.
__device__ __forceinline__ bool grid_sync(StepCtl *ctl, unsigned target, int where, int *sh_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&ctl->count, 1u);
        int ok = 1;
        long long t0 = 0;
        for (unsigned it = 0;; it++) {
            if ((int)(ld_acquire_u32(&ctl->count) - target) >= 0) break;
            if ((it & 31) == 31) {
                if (*(volatile int *)&ctl->abort) {
                    ok = 0;
                    break;
                }
                const long long t = globaltimer_ns();
                if (!t0) t0 = t;
                else if (t - t0 > g_step_wait_ns) {
                    atomicExch(&ctl->where, where + 1);
                    atomicExch(&ctl->abort, 1);
                    ok = 0;
                    break;
                }
            }
        }
        __threadfence();
        *sh_ok = ok;
    }
    __syncthreads();
    return *sh_ok != 0;
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
    t0 = (int)((long long)cid * a.RT / a.NC);
    t1 = (int)((long long)(cid + 1) * a.RT / a.NC);
    const int Uc = (t1 - t0) * a.KB;
    w0 = (int)((long long)Uc * wid / WARPS);
    w1 = (int)((long long)Uc * (wid + 1) / WARPS);
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

// One GEMV op (the body of k_gemv_tiled with clusters of one CTA): this CTA
// owns row tiles [t0, t1) whole, so every tile is finished here.
template <int QT>
__device__ __forceinline__ bool gemv_op(uint8_t *smem, const TArgs &a, Ring &r, const DOp *next, StepCtl *ctl) {
    constexpr int NB = 2, UNIT = unit_bytes(QT);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int w0, w1, t0, t1;
    const bool mine = warp_units(a, blockIdx.x, wid, w0, w1, t0, t1);
    const Smem<1, QT> L{a.KB, a.XL, a.maxrt, 0};
    float *acc = reinterpret_cast<float *>(smem + L.acc_off());
    bool ok = true;
    if (mine) {
        for (int i = threadIdx.x; i < a.maxrt * NB * 16; i += NTHR) acc[i] = 0.0f;
        build_x<1, QT, 0, true>(smem, L, a);
        __syncthreads();
        const float *inv = reinterpret_cast<const float *>(smem + L.sc_off()) + 8;
        const int XS = a.XL * XSTR, KB = a.KB;
        const uint8_t *xbl = smem + lane * XSTR;
        const uint32_t *xml = reinterpret_cast<const uint32_t *>(smem + L.xm_off()) + lane;
        const uint8_t *wbase = a.w + (size_t)t0 * KB * UNIT;
        Part<1> p;
        p.zero();
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
                if (cur >= 0) flush<1>(p, acc + cur * NB * 16, inv, a.nb, lane);
                p.zero();
                cur = rt;
            }
            const uint8_t *u = r.slots + (size_t)s * SLOT;
            const uint8_t *xb = xbl + kb * XS;
            if (QT == 4) unit_q4k<1>(p, u, xb, XS, xml + kb * 32, lane);
            else if (QT == 6) unit_q6k<1>(p, u, xb, XS, xml + kb * 32, lane);
            else unit_q80<1>(p, u, xb, XS, lane);
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
        if (cur >= 0 && ok) flush<1>(p, acc + cur * NB * 16, inv, a.nb, lane);
    }
    if (!ok) {
        atomicExch(&ctl->abort, 1);
    } else if (next) {
        // this warp's slots are all consumed: start the next GEMV's weights
        ring_prefill(r, next->g, next->qt, lane, wid);
    }
    if (!mine) return ok;
    __syncthreads();
    unsigned long long best[4] = {0ull, 0ull, 0ull, 0ull};
    for (int T = wid; T < t1 - t0; T += WARPS) epilogue_tile(a, (t0 + T) * 16, acc + T * NB * 16, lane, best);
    if (a.keys) {  // greedy keys: half-warp maxima, then one atomic per CTA and batch row
        auto kbest = reinterpret_cast<unsigned long long(*)[8]>(smem);
        __syncthreads();  // the x fragments at offset 0 are dead
#pragma unroll
        for (int j = 0; j < 4; j++) {
            unsigned long long k = best[j];
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
                k = o > k ? o : k;
            }
            if ((lane & 15) == 0) kbest[wid][2 * j + (lane >> 4)] = k;
        }
        __syncthreads();
        if ((int)threadIdx.x < a.nb) {
            unsigned long long k = 0ull;
            for (int w = 0; w < WARPS; w++) k = kbest[w][threadIdx.x] > k ? kbest[w][threadIdx.x] : k;
            if (k) atomicMax(a.keys + threadIdx.x, k);
        }
    }
    return ok;
}

// Attention work items (split, kv head, sequence), dealt round-robin to the
// CTAs; the last split of each (sequence, kv head) to finish merges them.
template <typename KV, int DH>
__device__ __forceinline__ void attn_op(uint8_t *smem, const AttnArgs &a, int items, int *sh_last) {
    const int G = a.H / a.Hkv, Dh = a.Dh, CH = a.CH;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int sp = it % a.nsplit, r2 = it / a.nsplit, kh = r2 % a.Hkv, b = r2 / a.Hkv;
        const int pos = __ldcg(a.pos + b);
        if (pos < 0 || pos >= a.S) continue;  // the host validates positions
        const int t0 = sp * CH, t1 = min(t0 + CH, pos + 1);
        if (t0 > pos) continue;
        float *wsb = a.ws + (((size_t)b * a.H + (size_t)kh * G) * a.nsplit + sp) * (Dh + 2);
        const size_t hstride = (size_t)a.nsplit * (Dh + 2);
        split_body<KV, DH, NTHR, 128>(a, reinterpret_cast<float *>(smem), sp, kh, b, pos, t0, t1, wsb, hstride);
        if (a.nsplit > 1) attn_merge_last<NTHR>(a, wsb, hstride, kh, b, pos, sh_last);
        __syncthreads();  // shared memory is reused by the next item
    }
}

template <int T>
__device__ __forceinline__ void embed_row(const EmbedArgs &e, int b) {
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
            }
        }
    }
}

__device__ __forceinline__ void embed_op(const EmbedArgs &e, int nb) {
    for (int b = blockIdx.x; b < nb; b += gridDim.x) {
        switch (e.type) {
        case LMC_TYPE_Q4_K: embed_row<LMC_TYPE_Q4_K>(e, b); break;
        case LMC_TYPE_Q6_K: embed_row<LMC_TYPE_Q6_K>(e, b); break;
        case LMC_TYPE_Q8_0: embed_row<LMC_TYPE_Q8_0>(e, b); break;
        case LMC_TYPE_F16: embed_row<LMC_TYPE_F16>(e, b); break;
        default: embed_row<LMC_TYPE_F32>(e, b); break;
        }
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
    __shared__ __align__(16) DOp op;
    __shared__ int sh_ok, sh_last;
    __shared__ unsigned sh_base;
    StepCtl *ctl = P.ctl;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        sh_ok = *(volatile int *)&ctl->abort == 0;  // an earlier launch gave up: run nothing
        sh_base = *(volatile unsigned *)&ctl->base;
    }
    __syncthreads();
    if (!sh_ok) return;
    const unsigned base = sh_base;
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
    if (P.first_gemv >= 0) ring_prefill(r, P.ops[P.first_gemv].g, P.ops[P.first_gemv].qt, lane, wid);
    unsigned passed = 0;
    bool alive = true;
    for (int i = 0; i < P.nops && alive; i++) {
        {  // this op's arguments into shared memory
            const int4 *src = reinterpret_cast<const int4 *>(P.ops + i);
            int4 *dst = reinterpret_cast<int4 *>(&op);
            for (int w = threadIdx.x; w < (int)(sizeof(DOp) / 16); w += NTHR) dst[w] = __ldg(src + w);
        }
        __syncthreads();
        const DOp *next = op.next_gemv >= 0 ? P.ops + op.next_gemv : nullptr;
        switch (op.kind) {
        case LMC_OP_EMBED: embed_op(op.e, op.nb); break;
        case LMC_OP_GEMV:
            if (op.qt == 4) alive = gemv_op<4>(smem, op.g, r, next, ctl);
            else if (op.qt == 6) alive = gemv_op<6>(smem, op.g, r, next, ctl);
            else alive = gemv_op<8>(smem, op.g, r, next, ctl);
            break;
        case LMC_OP_ATTN:
            if (op.kv == 0) {
                if (op.dh == 64) attn_op<float, 64>(smem, op.at, op.items, &sh_last);
                else attn_op<float, 128>(smem, op.at, op.items, &sh_last);
            } else {
                if (op.dh == 64) attn_op<__half, 64>(smem, op.at, op.items, &sh_last);
                else attn_op<__half, 128>(smem, op.at, op.items, &sh_last);
            }
            break;
        case LMC_OP_SAMPLE: sample_op(smem, op.sm, op.nb); break;
        default: advance_op(op.v, op.nb); break;
        }
        // a ring wait that ran out in any warp of any CTA aborts the step at
        // the next barrier (grid_sync polls the flag)
        if (op.sync) {
            passed++;
            alive = grid_sync(ctl, base + passed * gridDim.x, i, &sh_ok) && alive;
        }
        __syncthreads();  // every warp is done with `op` before it is replaced
    }
    if (alive && blockIdx.x == 0 && threadIdx.x == 0) ctl->base = base + passed * gridDim.x;
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

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct lmc_step_prog {
    DOp *d_ops;
    int nops, first_gemv, grid, stages, ring_off;
    size_t smem;
    StepCtl *ctl;
};

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
    a.NC = std::min(grid, a.RT);
    a.maxrt = (a.RT + a.NC - 1) / a.NC + 1;
    a.stages = stages;
    const int qt = qt_of_type(t->type), unit = unit_bytes(qt);
    a.pf = (int)std::min<long long>(64, PF_BYTES / ((long long)a.NC * WARPS * unit));
    d->g = a;
    d->qt = qt;
    return gemv_smem(qt, a.KB, a.XL, a.maxrt);
}

static size_t plan_attn(const lmc_step_op *o, DOp *d) {
    if (!o->out || !o->q || !o->k_new || !o->v_new || !o->k_cache || !o->v_cache || !o->pos || !o->cnt) return 0;
    if (o->batch <= 0 || o->H <= 0 || o->Hkv <= 0 || o->H % o->Hkv || (o->Dh != 64 && o->Dh != 128) || o->S <= 0)
        return 0;
    if (o->kv_dtype != LMC_KV_F32 && o->kv_dtype != LMC_KV_F16) return 0;
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
    d->kv = o->kv_dtype == LMC_KV_F16;
    d->dh = o->Dh;
    d->items = a.nsplit * o->Hkv * o->batch;
    const int G = o->H / o->Hkv;
    return (size_t)(G * o->Dh + G * a.CH + 2 * G + WARPS * ATT_GROUP * o->Dh) * sizeof(float);
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
                                   ops[i].V, ops[i].S, (int)ty, ops[i].y};
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
                                 ops[i].prompt, ops[i].n_prompt, ops[i].n_new, ops[i].kind == LMC_OP_ADVANCE,
                                 ops[i].from_next};
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
        if (d[i].kind == LMC_OP_GEMV) nxt = i;
        first = nxt;
    }
    lmc_step_prog *p = (lmc_step_prog *)calloc(1, sizeof(lmc_step_prog));
    if (!p) return lmc_set_error(LMC_ERR_OOM, "step_prog: host");
    p->nops = n;
    p->first_gemv = first;
    p->grid = grid;
    p->stages = stages;
    p->ring_off = (int)below;
    p->smem = smem;
    cudaError_t e = cudaMalloc((void **)&p->d_ops, sizeof(DOp) * n);
    if (e == cudaSuccess) e = cudaMalloc((void **)&p->ctl, sizeof(StepCtl));
    if (e == cudaSuccess) e = cudaMemcpy(p->d_ops, d.data(), sizeof(DOp) * n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(p->ctl, 0, sizeof(StepCtl));
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

extern "C" int lmc_step_prog_launch(const lmc_step_prog *p, cudaStream_t s) {
    if (!p) return lmc_set_error(LMC_ERR_INVALID, "step_prog_launch: null");
    StepParams P;
    P.ops = p->d_ops;
    P.nops = p->nops;
    P.first_gemv = p->first_gemv;
    P.ring_off = p->ring_off;
    P.stages = p->stages;
    P.ctl = p->ctl;
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
        if (c.abort) {
            cudaMemset(p->ctl, 0, sizeof(StepCtl));
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
