// Next-token selection on the device: greedy argmax and temperature sampling over logits
// [B][V], so that a decode loop never brings its logits or tokens to the host.
//
// The reference picks the next token on the host after every step: np.argmax over the
// logits row (src/mojollama/kernels/turbo_engine_v7_moe.py:2101-2114); its C engine has
// no sampler.  Greedy here is exactly np.argmax: the first maximum wins, and a NaN counts
// as the maximum (the first NaN wins).  Temperature sampling uses the Gumbel-max
// construction: token = argmax_i (logit_i / T + g_i), g_i = -log(-log u_i), which draws
// from softmax(logit / T) in one pass with no normalisation.  u_i comes from a
// counter-based generator (the SplitMix64 finaliser of Steele, Lea & Flood, 2014) keyed
// by (seed, step, row, i), so a draw is reproducible on any device or on the host
// (oracle/sampling.py restates it in numpy).
//
// Work split: each row is cut into chunks of kChunk logits; CTA (chunk, row) reduces its
// chunk to one 64-bit key (order-preserving bits of the score above, ~index below, so
// the larger score and then the smaller index wins) and folds it into the row's key with
// atomicMax.  The last CTA of a row to finish (arrival counter) writes the token and
// resets the row's key and counter to zero for the next call.  Bound: the logits read
// once (B * V * 4 bytes); MUFU throughput when sampling.
#include <cuda_runtime.h>
#include <math.h>

#include "../../include/mojollama_b200_ref_abi.h"
#include "mlq_internal.h"

namespace mlq {

constexpr int kSampleThreads = 256;
constexpr int kChunk = 4096;          // logits per CTA
constexpr int kSampleMaxRows = 1024;  // rows per call (persistent per-device state)

__host__ __device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// uniform in (0, 1) with 23 random bits: (j + 1/2) 2^-23 needs 24 significant bits, so it
// is exact in fp32 and strictly below 1 (with 24 bits, j + 1/2 near 2^24 would round up to
// 2^24, u to 1.0 and the Gumbel score to +inf)
__device__ __forceinline__ float sample_uniform(unsigned long long row_key, int i) {
    const unsigned long long h = mix64(row_key + 0x9E3779B97F4A7C15ull * (unsigned long long)(i + 1));
    return ((float)(h >> 41) + 0.5f) * 1.1920928955078125e-7f;   // 2^-23
}

// order-preserving 32-bit image of a float; every NaN maps to the top
__device__ __forceinline__ unsigned int order_key(float f) {
    if (isnan(f)) return 0xFFFFFFFFu;
    const unsigned int u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kSampleThreads) k_sample(const float *__restrict__ logits, int V, float inv_t,
                                                           int greedy, unsigned long long seed,
                                                           unsigned long long step, unsigned long long *best,
                                                           unsigned int *arrived, int *__restrict__ tokens) {
    const int b = blockIdx.y;
    const int lo = blockIdx.x * kChunk, hi = min(V, lo + kChunk);
    const float *row = logits + (size_t)b * V;
    const unsigned long long row_key = mix64(seed ^ mix64((step << 20) ^ (unsigned long long)b));
    unsigned long long key = 0;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float s = row[i];
        if (!greedy) s = s * inv_t - logf(-logf(sample_uniform(row_key, i)));
        const unsigned long long k = ((unsigned long long)order_key(s) << 32) | (0xFFFFFFFFu - (unsigned int)i);
        key = k > key ? k : key;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    __shared__ unsigned long long warp_best[kSampleThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) warp_best[warp] = key;
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < kSampleThreads / 32; w++) key = warp_best[w] > key ? warp_best[w] : key;
    atomicMax(&best[b], key);
    __threadfence();
    if (atomicAdd(&arrived[b], 1u) == gridDim.x - 1) {
        // last CTA of the row: every other CTA's atomicMax precedes its arrival
        const unsigned long long k = atomicExch(&best[b], 0ull);
        tokens[b] = (int)(0xFFFFFFFFu - (unsigned int)(k & 0xFFFFFFFFull));
        arrived[b] = 0u;
    }
}

// per-device row keys and arrival counters, zero between calls
struct SampleState {
    unsigned long long *best = nullptr;
    unsigned int *arrived = nullptr;
};
static SampleState g_sample[16];

static bool sample_state(int dev, SampleState *&st) {
    if (dev < 0 || dev >= 16) return false;
    st = &g_sample[dev];
    if (st->best) return true;
    void *p = nullptr;
    const size_t bytes = (size_t)kSampleMaxRows * (sizeof(unsigned long long) + sizeof(unsigned int));
    if (!MLQ_CUDA(cudaMalloc(&p, bytes))) return false;
    if (!MLQ_CUDA(cudaMemset(p, 0, bytes))) { cudaFree(p); return false; }
    st->best = static_cast<unsigned long long *>(p);
    st->arrived = reinterpret_cast<unsigned int *>(st->best + kSampleMaxRows);
    return true;
}

int launch_sample(const float *logits, int B, int V, float temperature, unsigned long long seed,
                  unsigned long long step, int *tokens, cudaStream_t s) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    SampleState *st = nullptr;
    if (!sample_state(c->device, st)) return mlq_last_error() ? mlq_last_error() : MLQ_ERR_CUDA;
    const int greedy = !(temperature > 0.0f);
    dim3 grid((unsigned)((V + kChunk - 1) / kChunk), (unsigned)B);
    k_sample<<<grid, kSampleThreads, 0, s>>>(logits, V, greedy ? 1.0f : 1.0f / temperature, greedy, seed, step,
                                             st->best, st->arrived, tokens);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

}  // namespace mlq

using namespace mlq;

extern "C" {

int mlq_sample(const float *logits, int B, int V, float temperature, unsigned long long seed,
               unsigned long long step, int *tokens) {
    if (!logits || !tokens || B <= 0 || V <= 0 || B > kSampleMaxRows) {
        set_error(MLQ_ERR_ARG, "mlq_sample: null pointer or sizes outside B 1..%d, V >= 1", kSampleMaxRows);
        return MLQ_ERR_ARG;
    }
    if (isnan(temperature) || isinf(temperature)) {
        set_error(MLQ_ERR_ARG, "mlq_sample: temperature must be finite (<= 0 selects greedy argmax)");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    const float *dl = (const float *)cs.in(logits, sizeof(float) * (size_t)B * V);
    int *dt = (int *)cs.out(tokens, sizeof(int) * (size_t)B);
    if (cs.failed) return cs.finish();
    int rc = launch_sample(dl, B, V, temperature, seed, step, dt, stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

int mlq_argmax(const float *logits, int B, int V, int *tokens) {
    return mlq_sample(logits, B, V, 0.0f, 0ull, 0ull, tokens);
}

// One decode step and its next tokens: batch_forward, then the sampler on the step's
// logits.  next_tokens may be the tokens buffer itself (both are consumed in stream order:
// the step copies its tokens before the sampler writes).  With device tokens, logits and
// next_tokens the whole call is asynchronous and nothing crosses to the host.
int mlq_batch_forward_sample(const void *bc, const int *tokens, int B, float *ws, float temperature,
                             unsigned long long seed, unsigned long long step, int *next_tokens) {
    if (!bc || !next_tokens) {
        set_error(MLQ_ERR_ARG, "mlq_batch_forward_sample: null model or next_tokens");
        return MLQ_ERR_ARG;
    }
    const int rc = mlq_batch_forward(bc, tokens, B, ws);
    if (rc != MLQ_OK) return rc;
    const BC *c = static_cast<const BC *>(bc);
    return mlq_sample(c->logits, B, c->outNR, temperature, seed, step, next_tokens);
}

}  // extern "C"
