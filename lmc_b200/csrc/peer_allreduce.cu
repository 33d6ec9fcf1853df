// peer_allreduce.cu - the tensor-parallel residual sum over peer memory.
//
// The column-split projections of a tensor-parallel layer leave each rank
// with a partial residual of B x D floats (16 KB per row at the 8B width),
// and the next op needs their sum on every rank.  An NCCL all-reduce of such
// a small message costs tens of microseconds at eight ranks, and a decode
// step has two per layer.  Here each rank owns a region of its own device
// memory that every peer maps (CUDA IPC, over NVLink / NVSwitch): a receive
// slot per peer and a flag per peer and chunk.  One launch per sum: CTA c
// takes chunk c (1024 floats), stores its partial into its slot on every
// peer with plain stores, raises its flag there (fenced at system scope),
// waits (bounded by %globaltimer) for every peer's flag of the same chunk on
// its own region, and adds the slots in rank order - the same order on
// every rank, so every rank ends with the same floats.  Slots and flags are
// double-buffered by the parity of a per-chunk sequence number (kept on the
// device, so the launch can live in a CUDA graph): a rank can only reuse a
// buffer after every peer has passed the following sum, which needs its own
// flags.  No multicast, no NVLS: plain peer loads and stores only.
#include "lmc_common.cuh"
#include "lmc_internal.h"

namespace {

constexpr int PEER_CHUNK = 1024;                       // floats per CTA
constexpr int PEER_MAXC = 128;                         // chunks: up to 131072 floats a sum
constexpr int PEER_MAXN = PEER_CHUNK * PEER_MAXC;
constexpr int PEER_THREADS = PEER_CHUNK / 4;           // one float4 per thread

// Region layout (bytes), the same on every rank:
//   recv  [2][LMC_PEER_MAX][PEER_MAXN] floats
//   flags [2][LMC_PEER_MAX][PEER_MAXC] u32   (flags[par][p][c]: peer p's chunk c arrived)
//   seq   [PEER_MAXC] u32                    (this rank's sequence number per chunk)
constexpr size_t RECV_BYTES = (size_t)2 * LMC_PEER_MAX * PEER_MAXN * 4;
constexpr size_t FLAG_OFF = RECV_BYTES, FLAG_BYTES = (size_t)2 * LMC_PEER_MAX * PEER_MAXC * 4;
constexpr size_t SEQ_OFF = FLAG_OFF + FLAG_BYTES, REGION_BYTES = SEQ_OFF + PEER_MAXC * 4;

struct PeerArgs {
    float *x;
    int n, rank, size;
    uint8_t *base[LMC_PEER_MAX];  // every rank's region (base[rank] = this rank's own)
};

__device__ long long g_peer_wait_ns = 1000000000ll;
__device__ int g_peer_err;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ long long gtimer() {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// base[p] for a runtime p without a local copy of the parameter array
__device__ __forceinline__ uint8_t *base_of(const PeerArgs &a, int p) {
    uint8_t *r = a.base[0];
#pragma unroll
    for (int k = 1; k < LMC_PEER_MAX; k++) r = p == k ? a.base[k] : r;
    return r;
}

__global__ void __launch_bounds__(PEER_THREADS) k_peer_allreduce(PeerArgs a) {
    pdl_wait();  // the partials are written by the previous kernels
    pdl_launch_dependents();
    const int c = blockIdx.x, tid = threadIdx.x;
    const int i = c * PEER_CHUNK + 4 * tid;
    uint8_t *const own_base = base_of(a, a.rank);
    unsigned *seq = reinterpret_cast<unsigned *>(own_base + SEQ_OFF) + c;
    __shared__ unsigned sh_s;
    if (tid == 0) sh_s = *seq + 1;
    __syncthreads();
    const unsigned s = sh_s, par = s & 1;
    const bool live = i < a.n;
    const float4 mine = live ? *reinterpret_cast<const float4 *>(a.x + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    // 1. my partial into my slot on every peer
#pragma unroll
    for (int p = 0; p < LMC_PEER_MAX; p++) {
        if (p >= a.size) break;
        if (p == a.rank || !live) continue;
        float *slot = reinterpret_cast<float *>(a.base[p]) + ((size_t)par * LMC_PEER_MAX + a.rank) * PEER_MAXN;
        *reinterpret_cast<float4 *>(slot + i) = mine;
    }
    __syncthreads();
    // 2. my flag of this chunk on every peer (release at system scope: the
    //    CTA's stores above are ordered before it by the barrier)
    if (tid < a.size && tid != a.rank) {
        unsigned *f = reinterpret_cast<unsigned *>(base_of(a, tid) + FLAG_OFF) +
                      ((size_t)par * LMC_PEER_MAX + a.rank) * PEER_MAXC + c;
        st_release_sys(f, s);
    }
    // 3. every peer's flag of this chunk on my region (bounded wait)
    __shared__ int sh_ok;
    if (tid == 0) sh_ok = 1;
    __syncthreads();
    if (tid < a.size && tid != a.rank) {
        const unsigned *f = reinterpret_cast<const unsigned *>(own_base + FLAG_OFF) +
                            ((size_t)par * LMC_PEER_MAX + tid) * PEER_MAXC + c;
        long long t0 = 0;
        for (unsigned it = 0;; it++) {
            if ((int)(ld_acquire_sys(f) - s) >= 0) break;
            if ((it & 63) == 63) {
                const long long t = gtimer();
                if (!t0) t0 = t;
                else if (t - t0 > g_peer_wait_ns) {
                    atomicExch(&g_peer_err, 1);
                    sh_ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    // 4. the sum in rank order (identical on every rank)
    if (live && sh_ok) {
        const float *own = reinterpret_cast<const float *>(own_base);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < a.size; p++) {
            float4 v = mine;
            if (p != a.rank) v = __ldcg(reinterpret_cast<const float4 *>(own + ((size_t)par * LMC_PEER_MAX + p) * PEER_MAXN + i));
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        *reinterpret_cast<float4 *>(a.x + i) = acc;
    }
    if (tid == 0) *seq = s;
}

}  // namespace

extern "C" size_t lmc_peer_region_bytes(void) { return REGION_BYTES; }

extern "C" int lmc_peer_max_floats(void) { return PEER_MAXN; }

extern "C" int lmc_peer_allreduce(float *d_x, int n, int rank, int size, void *const *bases, cudaStream_t s) {
    if (!d_x || n <= 0 || n > PEER_MAXN || (n & 3) || ((uintptr_t)d_x & 15) || size < 2 || size > LMC_PEER_MAX ||
        rank < 0 || rank >= size || !bases)
        return lmc_set_error(LMC_ERR_INVALID, "peer allreduce: n %d, rank %d of %d", n, rank, size);
    PeerArgs a;
    a.x = d_x;
    a.n = n;
    a.rank = rank;
    a.size = size;
    for (int p = 0; p < LMC_PEER_MAX; p++) a.base[p] = p < size ? (uint8_t *)bases[p] : nullptr;
    for (int p = 0; p < size; p++)
        if (!a.base[p]) return lmc_set_error(LMC_ERR_INVALID, "peer allreduce: region of rank %d missing", p);
    LMC_LAUNCH("peer allreduce", k_peer_allreduce, (n + PEER_CHUNK - 1) / PEER_CHUNK, PEER_THREADS, 0, s, a);
    return LMC_OK;
}

// LMC_OK, or LMC_ERR_TIMEOUT once after a peer sum gave up waiting for a
// peer (a rank that stopped); the flag is cleared.
extern "C" int lmc_peer_status(void) {
    int v = 0;
    LMC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_peer_err, sizeof(int)));
    if (!v) return LMC_OK;
    const int zero = 0;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_peer_err, &zero, sizeof(int)));
    return lmc_set_error(LMC_ERR_TIMEOUT, "a peer sum gave up waiting for a rank");
}

extern "C" int lmc_peer_set_wait_limit(long long ns) {
    const long long v = ns > 0 ? ns : 1000000000ll;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_peer_wait_ns, &v, sizeof v));
    return LMC_OK;
}
