// Log-mel spectrogram on the device (mel.logMel, src/mel.zig:103-157): 16 kHz samples, 200
// samples reflected at the front and 30 s of zeros appended, 400-sample periodic Hann
// frames every 160 samples, the power of the 201 DFT bins, the model's mel filters, log10
// with a 1e-10 floor, then the clamp to (max - 8) and (x + 4) / 4.
//
// mel_tables_kernel: the Hann window and the cos / sin tables of the 400-point DFT, computed in
//   f64 and rounded to f32 as the reference's tables are.
// mel_frames_kernel: one block per 16 frames. The windowed frames go to shared memory with
//   the tables; each thread owns one DFT bin for the 16 frames (f32 sums over the 400
//   samples, the table index stepping by the bin number modulo 400; the reference reaches
//   the same sums through a radix-2 split into 25-point DFTs, so results agree to f32
//   rounding, not bit for bit), power = re^2 + im^2 in f32; then each (frame, filter) pair
//   sums power x filter in f64 and takes log10 in f64, as the reference does. Frames past
//   the audio (and its front pad) hold log10(1e-10). Each block folds its maximum into one
//   word (an order-preserving integer image of the float).
// mel_clamp_kernel: v = max(v, max - 8) (compared in f64), then (v + 4) / 4 in f32.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zwg {

namespace mel {
constexpr int N_FFT = 400;
constexpr int HOP = 160;
constexpr int N_BINS = N_FFT / 2 + 1;  // 201
constexpr int PAD_FRONT = N_FFT / 2;   // 200
constexpr int FB = 16;                 // frames per block
constexpr int THREADS = 224;           // >= N_BINS

// Order-preserving map of f32 onto u32 (larger float, larger integer).
__device__ __forceinline__ uint32_t ordered(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unordered(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
}  // namespace mel

__global__ void mel_tables_kernel(float* tables) {
    using namespace mel;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N_FFT) return;
    const double x = 2.0 * 3.14159265358979323846 * (double)i / (double)N_FFT;
    tables[i] = (float)(0.5 - 0.5 * cos(x));  // periodic Hann
    tables[N_FFT + i] = (float)cos(x);
    tables[2 * N_FFT + i] = (float)sin(x);
}

__global__ void __launch_bounds__(mel::THREADS) mel_frames_kernel(const float* __restrict__ samples, long long n,
                                                                  const float* __restrict__ tables,
                                                                  const float* __restrict__ filters, int n_mel,
                                                                  long long n_len, long long n_frames_real,
                                                                  float* __restrict__ out, uint32_t* max_word) {
    using namespace mel;
    __shared__ float frame[FB][N_FFT];
    __shared__ float cs[N_FFT], sn[N_FFT];
    __shared__ float power[FB][N_BINS + 1];
    __shared__ uint32_t blk_max;
    const long long f0 = (long long)blockIdx.x * FB;
    const long long n_real = n + PAD_FRONT;
    if (threadIdx.x == 0) blk_max = 0;
    for (int i = threadIdx.x; i < N_FFT; i += THREADS) {
        cs[i] = tables[N_FFT + i];
        sn[i] = tables[2 * N_FFT + i];
    }
    // windowed frames: padded[p] = samples[200 - p] (reflection) for p < 200, samples[p - 200]
    // for the audio, zero past it
    for (int e = threadIdx.x; e < FB * N_FFT; e += THREADS) {
        const int f = e / N_FFT, j = e - f * N_FFT;
        const long long fi = f0 + f;
        float v = 0.f;
        if (fi < n_frames_real) {
            const long long p = fi * HOP + j;
            float x = 0.f;
            if (p < PAD_FRONT) {
                const long long src = PAD_FRONT - p;
                if (p + 1 < n && src < n) x = samples[src];
            } else if (p < n_real) {
                x = samples[p - PAD_FRONT];
            }
            v = tables[j] * x;
        }
        frame[f][j] = v;
    }
    __syncthreads();
    // one DFT bin per thread over the block's frames
    const int k = threadIdx.x;
    if (k < N_BINS) {
        float re[FB], im[FB];
#pragma unroll
        for (int f = 0; f < FB; f++) re[f] = im[f] = 0.f;
        int idx = 0;
        for (int j = 0; j < N_FFT; j++) {
            const float c = cs[idx], s = sn[idx];
#pragma unroll
            for (int f = 0; f < FB; f++) {
                re[f] = fmaf(frame[f][j], c, re[f]);
                im[f] = fmaf(-frame[f][j], s, im[f]);
            }
            idx += k;
            if (idx >= N_FFT) idx -= N_FFT;
        }
#pragma unroll
        for (int f = 0; f < FB; f++) power[f][k] = __fadd_rn(__fmul_rn(re[f], re[f]), __fmul_rn(im[f], im[f]));
    }
    __syncthreads();
    // mel filters: f64 sums of f32 products, log10 with the 1e-10 floor
    float lmax = -INFINITY;
    for (int e = threadIdx.x; e < FB * n_mel; e += THREADS) {
        const int f = e / n_mel, c = e - f * n_mel;
        const long long fi = f0 + f;
        if (fi >= n_len) continue;
        float v;
        if (fi < n_frames_real) {
            const float* row = filters + (size_t)c * N_BINS;
            double sum = 0.0;
            for (int b = 0; b < N_BINS; b++) sum += (double)power[f][b] * (double)__ldg(row + b);
            v = (float)log10(fmax(sum, 1e-10));
        } else {
            v = (float)log10(1e-10);
        }
        out[(size_t)c * n_len + fi] = v;
        lmax = fmaxf(lmax, v);
    }
    lmax = warp_max(lmax);
    if ((threadIdx.x & 31) == 0 && lmax > -INFINITY) atomicMax(&blk_max, ordered(lmax));
    __syncthreads();
    if (threadIdx.x == 0 && blk_max) atomicMax(max_word, blk_max);
}

__global__ void mel_clamp_kernel(float* data, long long count, const uint32_t* max_word) {
    using namespace mel;
    const double mmax = (double)unordered(*max_word) - 8.0;
    const float fmx = (float)mmax;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x) {
        float v = data[i];
        if ((double)v < mmax) v = fmx;
        data[i] = (v + 4.0f) / 4.0f;
    }
}

size_t mel_frames(size_t n_samples) { return (n_samples + 16000 * 30) / mel::HOP; }

size_t mel_scratch_bytes() { return 256 + 3 * mel::N_FFT * sizeof(float); }

int log_mel_launch(const float* samples, size_t n, const float* filters, int n_mel, float* out, void* scratch,
                   int sm_count, cudaStream_t st) {
    using namespace mel;
    if (n == 0 || n_mel <= 0) return -1;
    const long long n_len = (long long)mel_frames(n);
    const long long n_real = (long long)n + PAD_FRONT;
    const long long n_frames_real = std::min<long long>(n_real / HOP + 1, n_len);
    uint32_t* max_word = static_cast<uint32_t*>(scratch);
    float* tables = reinterpret_cast<float*>(static_cast<char*>(scratch) + 256);
    if (cudaMemsetAsync(max_word, 0, sizeof(uint32_t), st) != cudaSuccess) return -1;
    mel_tables_kernel<<<(N_FFT + 127) / 128, 128, 0, st>>>(tables);
    const long long blocks = (n_len + FB - 1) / FB;
    if (blocks > 0x7fffffff) return -1;
    mel_frames_kernel<<<(unsigned)blocks, THREADS, 0, st>>>(samples, (long long)n, tables, filters, n_mel, n_len,
                                                           n_frames_real, out, max_word);
    const long long count = n_len * n_mel;
    const int grid = (int)std::min<long long>((count + 255) / 256, 8LL * std::max(1, sm_count));
    mel_clamp_kernel<<<grid, 256, 0, st>>>(out, count, max_word);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace zwg
