// matvec.cuh -- dequant-matvec job descriptors shared by matvec.cu and the
// ABI layer.
#pragma once

#include "common.cuh"

#define DS4F_FMT_MLX4 1
#define DS4F_FMT_BF16 3

namespace ds4f {

// One y = W x. Formats and their reference counterparts:
//   FP8   W: E4M3 bytes [R x C]; s: [SR x SC] block scales, E8M0 bytes
//         (ds4f_f8_matvec, src/kernels.c:243-270) or fp32 (BASELINE);
//         element (r, c) uses s[r*SR/R][c*SC/C].
//   MXFP4 W: E2M1 nibbles, flat index i = r*C + c, byte i>>1, even i low
//         nibble; s: E8M0 byte per bsize flat elements
//         (ds4f_mxfp4_matvec, src/kernels.c:48-62).
//   BF16  W: bf16 [R x C]; s: optional fp32 bias [R]
//         (ds4f_bf16_matvec, src/kernels.c:91-103).
//   MLX4  W: u32 words of 8 nibbles, flat element k = (v[k/8] >> 4(k%8)) &
//         15; s, b: bf16 scale and bias per 64 flat elements; element =
//         q*s + b (ds4f_mlx4_matvec, src/kernels.c:154-222).
struct MvJob {
    const void *v;
    const void *s;
    const void *b;    // MLX4 biases (may be null)
    const float *x;
    float *y;
    int R, C, SR, SC;
    int fmt;
    int scale_kind;   // FP8: DS4F_SCALE_E8M0 / DS4F_SCALE_F32
    int bsize;        // MXFP4: 16 or 32
    int canon;        // FP8: apply the e=15 -> 448 rule in-kernel
    int fast;         // set by plan_jobs: shape fits the vector path
    int item0;        // first work item (prefix over jobs)
    int lpr;          // lanes per row in the vector path
    int nq;           // 16-byte chunks per row
    int streamed;     // taken by the TMA stream kernel (mvstream.cu), not by k_mv_jobs
};

// The stream kernel's work: units of up to 64 rows of one job (<= 32 KB),
// CTA c taking units [ranges[c], ranges[c+1]).
struct MvUnit {
    int job, row0, nrows, bytes;
};
struct MvStream {
    void *base;
    MvUnit *units;
    int *ranges;
    unsigned *err;    // set when a copy wait gave up
    int nunits, grid;
};
// Host: mark the jobs the stream kernel takes (J.streamed; expert-shaped
// FP8 / MXFP4 / BF16 rows of 128..2048 columns, 16-byte aligned) and upload
// its units, balanced by bytes over the SMs. plan_jobs then leaves them out.
int stream_plan(MvJob *jobs, int njobs, MvStream *sp);
void stream_free(MvStream *sp);
int stream_launch(const MvJob *jobs_dev, const MvStream &sp, cudaStream_t st);
// Synchronous: -1 if a copy wait of an earlier launch gave up (then cleared).
int stream_check(const MvStream &sp);

// Host: fill fast/lpr/nq/item0 and return the total work items.
int plan_jobs(MvJob *jobs, int njobs);
// Launch all jobs (device pointers inside jobs_dev) on one stream.
int launch_jobs(const MvJob *jobs_dev, int njobs, int nitems, cudaStream_t st);
// Element-exact dequantisation dumps (the "bit-exact dequantised weights"
// parity object): FP8 rows [r0, r1) -> fp32, MXFP4 flat [0, n) -> fp32.
int launch_f8_decode(const uint8_t *W, int scale_kind, const void *scales,
                     int R, int C, int SR, int SC, int r0, int r1, float *out,
                     cudaStream_t st);
int launch_mx_decode(const uint8_t *vals, const uint8_t *scales, int64_t n,
                     int bsize, float *out, cudaStream_t st);
// In-place e=15 canonicalisation of an E4M3 byte buffer (pool load).
int launch_f8_canon(uint8_t *buf, int64_t n, cudaStream_t st);

constexpr int kMvRowsPerItem = 64;
constexpr int kMvThreads = 256;

}  // namespace ds4f
