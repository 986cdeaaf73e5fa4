// encode_static.cu -- the arithmetic encoder with its scratch memory in a fixed
// device array, for callers that may not allocate device memory.
//
// Same coder as k_encode (rust/src/arith_coder.rs:8-136: interval update,
// E1/E2/E3 renormalisation with pending bits, MSB-first packing, finish = one
// '1' bit and a zero-padded last byte), but every buffer it needs between its
// inputs and its outputs -- the per-chunk output slots, their offsets, the
// encoded lengths and an error word -- lives in g_encode_scratch, a file-scope
// __device__ array of kStaticScratchBytes.  The entry point calls no cudaMalloc
// or cudaFree and nothing that allocates.  Every GPU that loads the library
// holds the array until the process exits.
//
// In host code g_encode_scratch is only a host-side stand-in for the device
// array, so it is never passed to a kernel.  The first call on a device (with
// that device current) looks up the array's device address with
// cudaGetSymbolAddress and keeps it, together with the CUDA context it belongs
// to, for later calls on that device; a call in a newer context (after a
// cudaDeviceReset) looks it up again.  Make the first call on each device, and
// the first after a reset, before any stream capture.  All calls share the one array, which
// keeps the previous call's contents: each call clears what must start at zero.
// Calls whose work overlaps on the GPU (other streams, other host threads) race
// on the array and must be serialised by the caller.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "czg.h"

namespace czg {
namespace {

constexpr uint64_t kStaticScratchBytes = 12ull << 20;
constexpr uint32_t kMaxChunks = CZG_STATIC_MAX_CHUNKS;
constexpr uint64_t kMaxTokens = CZG_STATIC_MAX_TOKENS;
// layout: [0] error word, [1] total packed bytes; then slot offsets (u64 x
// kMaxChunks+1), lengths (u32 x kMaxChunks), pack offsets (u64 x kMaxChunks+1),
// row offsets (u64 x kMaxChunks+1), then the slot bytes.
constexpr uint64_t kOffSlot = 16;
constexpr uint64_t kOffLens = kOffSlot + 8ull * (kMaxChunks + 1);
constexpr uint64_t kOffPack = kOffLens + 4ull * kMaxChunks;
constexpr uint64_t kOffRow = kOffPack + 8ull * (kMaxChunks + 1);
constexpr uint64_t kOffBytes = (kOffRow + 8ull * (kMaxChunks + 1) + 255) & ~255ull;
static_assert(kOffBytes + 4 * kMaxTokens + 8ull * kMaxChunks <= kStaticScratchBytes,
              "static scratch too small for its stated limits");

__device__ __align__(256) uint8_t g_encode_scratch[kStaticScratchBytes];

constexpr int kErrCap = 1, kErrSlot = 2, kErrSum = 4;

struct Scratch {
    uint32_t *err;
    uint64_t *total;
    uint64_t *slot_off;
    uint32_t *lens;
    uint64_t *pack_off;
    uint64_t *row_off;
    uint8_t *bytes;
};

__host__ __device__ inline Scratch scratch_at(uint8_t *base) {
    Scratch s;
    s.err = reinterpret_cast<uint32_t *>(base);
    s.total = reinterpret_cast<uint64_t *>(base + 8);
    s.slot_off = reinterpret_cast<uint64_t *>(base + kOffSlot);
    s.lens = reinterpret_cast<uint32_t *>(base + kOffLens);
    s.pack_off = reinterpret_cast<uint64_t *>(base + kOffPack);
    s.row_off = reinterpret_cast<uint64_t *>(base + kOffRow);
    s.bytes = base + kOffBytes;
    return s;
}

// Exclusive scans of the chunk lengths: rows and slot bytes (4*len + 8); one CTA.
// Lengths that do not add up to n_tokens (the caller's interval count) set kErrSum,
// and the kernels after this one then read no interval and write no output.
__global__ void k_static_layout(const uint32_t *__restrict__ chunk_len, uint32_t n, uint64_t n_tokens,
                                uint8_t *base) {
    Scratch s = scratch_at(base);
    __shared__ uint64_t carry_rows, carry_slot;
    if (threadIdx.x == 0) {
        carry_rows = 0;
        carry_slot = 0;
        *s.err = 0;
        *s.total = 0;
    }
    __syncthreads();
    for (uint32_t b = 0; b < n; b += blockDim.x) {
        const uint32_t i = b + threadIdx.x;
        const uint64_t len = i < n ? chunk_len[i] : 0;
        // block-wide inclusive scan (Hillis-Steele in shared memory)
        __shared__ uint64_t sr[1024], ss[1024];
        sr[threadIdx.x] = len;
        ss[threadIdx.x] = i < n ? 4 * len + 8 : 0;
        __syncthreads();
        for (uint32_t o = 1; o < blockDim.x; o <<= 1) {
            uint64_t ar = threadIdx.x >= o ? sr[threadIdx.x - o] : 0;
            uint64_t as = threadIdx.x >= o ? ss[threadIdx.x - o] : 0;
            __syncthreads();
            sr[threadIdx.x] += ar;
            ss[threadIdx.x] += as;
            __syncthreads();
        }
        if (i < n) {
            s.row_off[i] = carry_rows + sr[threadIdx.x] - len;
            s.slot_off[i] = carry_slot + ss[threadIdx.x] - (4 * len + 8);
            s.lens[i] = 0;
        }
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) {
            carry_rows += sr[threadIdx.x];
            carry_slot += ss[threadIdx.x];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        s.row_off[n] = carry_rows;
        s.slot_off[n] = carry_slot;
        if (carry_rows != n_tokens) *s.err = kErrSum;
    }
}

struct StaticSink {
    uint8_t *out;
    uint32_t cap, len;
    unsigned long long acc;
    int n;
    bool overflow;
    __device__ __forceinline__ void push(uint32_t bits, int count) {   // count <= 32
        acc = (acc << count) | bits;
        n += count;
        while (n >= 8) {
            n -= 8;
            const uint8_t b = (uint8_t)(acc >> n);
            if (len < cap) out[len] = b; else overflow = true;
            len++;
        }
        acc &= (1ull << n) - 1ull;
    }
    __device__ __forceinline__ void bit_plus_pending(uint32_t bit, uint32_t run) {
        push(bit, 1);
        const uint32_t fill = bit ? 0u : 0xFFFFFFFFu;
        while (run > 0) {
            const int c = run > 32 ? 32 : (int)run;
            push(c == 32 ? fill : (fill & ((1u << c) - 1u)), c);
            run -= (uint32_t)c;
        }
    }
};

// one thread per chunk; intervals (sym_low, sym_high) of the chunk's tokens
__global__ void k_static_encode(const uint2 *__restrict__ lohi, uint32_t n, uint32_t total,
                                unsigned long long inv_total, uint64_t slot_limit, uint8_t *base) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= n) return;
    Scratch s = scratch_at(base);
    if (*s.err & kErrSum) return;   // the row offsets would leave the caller's intervals
    const unsigned long long HALF = 1ull << 31, QUARTER = 1ull << 30, MASK = 0xFFFFFFFFull;
    const uint64_t r0 = s.row_off[c], cnt = s.row_off[c + 1] - r0;
    if (s.slot_off[c + 1] > slot_limit) {
        atomicOr(s.err, (uint32_t)kErrSlot);
        return;
    }
    StaticSink bs;
    bs.out = s.bytes + s.slot_off[c];
    bs.cap = (uint32_t)(s.slot_off[c + 1] - s.slot_off[c]);
    bs.len = 0;
    bs.acc = 0;
    bs.n = 0;
    bs.overflow = false;
    unsigned long long low = 0, high = MASK;
    uint32_t pending = 0;
    for (uint64_t i = 0; i < cnt; i++) {
        const uint2 lh = lohi[r0 + i];
        const unsigned long long range = high - low + 1;
        high = low + udiv_by_inv((unsigned long long)lh.y * range, total, inv_total) - 1;
        low = low + udiv_by_inv((unsigned long long)lh.x * range, total, inv_total);
        for (;;) {
            if (((low ^ high) & HALF) == 0) {
                bs.bit_plus_pending((uint32_t)((low >> 31) & 1ull), pending);
                pending = 0;
                low = (low << 1) & MASK;
                high = ((high << 1) & MASK) | 1ull;
            } else if ((low & ~high & QUARTER) != 0) {
                pending++;
                low = ((low << 1) ^ HALF) & MASK;
                high = (((high ^ HALF) << 1) | HALF | 1ull) & MASK;
            } else {
                break;
            }
        }
    }
    bs.push(1u, 1);
    if (bs.n > 0) bs.push(0u, 8 - bs.n);
    s.lens[c] = bs.len;
    if (bs.overflow) atomicOr(s.err, (uint32_t)kErrSlot);
}

// exclusive scan of the encoded lengths, then the total (one CTA)
__global__ void k_static_packoff(uint32_t n, uint8_t *base) {
    Scratch s = scratch_at(base);
    __shared__ uint64_t sv[1024];
    __shared__ uint64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (uint32_t b = 0; b < n; b += blockDim.x) {
        const uint32_t i = b + threadIdx.x;
        const uint64_t v = i < n ? s.lens[i] : 0;
        sv[threadIdx.x] = v;
        __syncthreads();
        for (uint32_t o = 1; o < blockDim.x; o <<= 1) {
            uint64_t a = threadIdx.x >= o ? sv[threadIdx.x - o] : 0;
            __syncthreads();
            sv[threadIdx.x] += a;
            __syncthreads();
        }
        if (i < n) s.pack_off[i] = carry + sv[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += sv[threadIdx.x];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        s.pack_off[n] = carry;
        *s.total = carry;
    }
}

// one CTA per chunk: slot bytes -> caller's packed output, lengths -> caller
__global__ void k_static_pack(uint32_t n, uint64_t out_cap, uint8_t *__restrict__ out,
                              uint32_t *__restrict__ out_lens, uint8_t *base) {
    Scratch s = scratch_at(base);
    const uint32_t c = blockIdx.x;
    if (*s.err & kErrSum) return;
    if (*s.total > out_cap) {
        if (c == 0 && threadIdx.x == 0) atomicOr(s.err, (uint32_t)kErrCap);
        return;
    }
    const uint32_t len = s.lens[c];
    const uint8_t *src = s.bytes + s.slot_off[c];
    uint8_t *dst = out + s.pack_off[c];
    for (uint32_t i = threadIdx.x; i < len; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) out_lens[c] = len;
}

// device address of g_encode_scratch, looked up once per device and context
// (cuCtxGetCurrent through the runtime's driver entry point: a cudaDeviceReset
// makes a new primary context, in which the array may sit elsewhere)
using CtxGetCurrentFn = int (*)(void **);

CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    }
    return fn;
}

std::mutex g_addr_mu;
uint8_t *g_addr[256] = {nullptr};
void *g_addr_ctx[256] = {nullptr};

int scratch_address(int dev, uint8_t **out) {
    if (dev < 0 || dev >= 256) return CZG_E_DEVICE;
    CtxGetCurrentFn get_ctx = ctx_get_current();
    if (!get_ctx) return CZG_E_DEVICE;
    std::lock_guard<std::mutex> lk(g_addr_mu);
    void *ctx = nullptr;
    if (get_ctx(&ctx) != 0) return CZG_E_DEVICE;
    if (!ctx) {   // no context current yet: cudaSetDevice makes the device's primary context current
        if (cudaSetDevice(dev) != cudaSuccess || get_ctx(&ctx) != 0 || !ctx) return CZG_E_DEVICE;
    }
    if (!g_addr[dev] || g_addr_ctx[dev] != ctx) {
        g_addr[dev] = nullptr;
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_encode_scratch) != cudaSuccess || !p) return CZG_E_DEVICE;
        g_addr[dev] = static_cast<uint8_t *>(p);
        g_addr_ctx[dev] = ctx;
    }
    *out = g_addr[dev];
    return CZG_OK;
}

}  // namespace
}  // namespace czg

extern "C" int czg_encode_intervals_static(const uint32_t *d_lohi, const uint32_t *d_chunk_len,
                                           uint32_t n_chunks, uint64_t n_tokens, uint32_t target_total,
                                           uint8_t *d_out, uint64_t out_cap, uint32_t *d_out_lens,
                                           uint64_t *out_bytes, void *stream) {
    using namespace czg;
    if (out_bytes) *out_bytes = 0;
    if (n_chunks == 0) return CZG_OK;
    if (!d_lohi || !d_chunk_len || !d_out || !d_out_lens || !out_bytes) return CZG_E_ARG;
    if (n_chunks > kMaxChunks || n_tokens > kMaxTokens) return CZG_E_LIMIT;
    if (target_total == 0) return CZG_E_ARG;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return CZG_E_DEVICE;
    uint8_t *base = nullptr;
    int st = scratch_address(dev, &base);
    if (st != CZG_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t slot_limit = kStaticScratchBytes - kOffBytes;
    k_static_layout<<<1, 1024, 0, s>>>(d_chunk_len, n_chunks, n_tokens, base);
    k_static_encode<<<(n_chunks + 127) / 128, 128, 0, s>>>(reinterpret_cast<const uint2 *>(d_lohi), n_chunks,
                                                           target_total, 0xFFFFFFFFFFFFFFFFull / target_total,
                                                           slot_limit, base);
    k_static_packoff<<<1, 1024, 0, s>>>(n_chunks, base);
    k_static_pack<<<n_chunks, 128, 0, s>>>(n_chunks, out_cap, d_out, d_out_lens, base);
    if (cudaGetLastError() != cudaSuccess) return CZG_E_DEVICE;
    uint64_t head[2] = {0, 0};   // error word, total bytes
    if (cudaMemcpyAsync(head, base, sizeof(head), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return CZG_E_DEVICE;
    const uint32_t err = (uint32_t)head[0];
    *out_bytes = head[1];
    if (err & kErrSum) {   // nothing was encoded or written
        *out_bytes = 0;
        return CZG_E_ARG;
    }
    if (err & kErrSlot) return CZG_E_LIMIT;   // chunk lengths summing past the stated limit
    if (err & kErrCap) return CZG_E_CAPACITY;
    return CZG_OK;
}
