// Host-visible description of one launch of the K-quant matvec family.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <string>

namespace si {

// How the input vector is formed in shared memory before the dot products.
enum XMode : int {
  XM_RAW = 0,      // x
  XM_RMS1P = 1,    // x * rsqrt(mean(x^2) + eps) * (1 + w)    (qwen35.rs:53-86, heads = 1)
  XM_GATED = 2,    // per head: c * rsqrt(mean(c^2) + eps) * w[d] * SiLU(z)  (qwen35.rs:14-49)
  XM_SIGGATE = 3,  // a / (1 + exp(-gate))                       (qwen35_runtime.rs:861-865)
};

struct QmvSeg {
  const uint8_t* w;     // row-major super-blocks of this segment
  float* y;             // output rows
  const float* resid;   // optional residual added in the epilogue (may alias y)
  uint32_t rows;
  uint32_t pad;
};

// Row-sharded output gathered by the matvec kernel itself over NVLink peer
// memory (mapped with CUDA IPC), with no fence on the data path: the epilogue
// stores each of this rank's rows into every rank's exchange words as one
// 8-byte word {value, launch epoch} (a single 64-bit store, so the value and
// its epoch land together), and every CTA then waits, bounded, for the words
// of its slice of the whole gathered vector to carry this launch's epoch and
// unpacks them into the float vector y. The words alternate between two
// parity halves (epoch & 1): a rank's launch k + 2 cannot start before every
// rank has finished launch k, so a word is never overwritten while it is
// still awaited. The epoch is this rank's count of launches on the buffer,
// read from `epoch` on the device (after the previous grid has finished) and
// advanced by the launch's last CTA, so a launch replayed from a CUDA graph
// synchronises like a fresh one.
constexpr int kPeerMax = 8;
struct PeerOut {
  uint32_t n;                 // ranks; 0 = ordinary output
  uint32_t rank;
  uint64_t* ll[kPeerMax];     // each rank's exchange words of the gathered vector (parity half 0)
  uint64_t parity_stride;     // words between the two parity halves
  float* y;                   // this rank's gathered vector (every rank's rows)
  uint32_t row0;              // this rank's first row in the gathered vector
  uint32_t total;             // rows of the gathered vector
  uint32_t* ticket;           // CTAs of the current launch that have finished (zero between launches)
  uint32_t* epoch;            // launches completed on this buffer by this rank
  long long wait_cycles;      // bound of each CTA's wait for the other ranks' rows
};

struct QmvParams {
  uint32_t type;        // SI_GGML_TYPE_Q4_K / Q5_K / Q6_K
  uint32_t cols;        // multiple of 256
  uint32_t nseg;        // 1..4 segments sharing x (grouped matvec)
  uint32_t pair;        // 1: SwiGLU, seg[0] = gate, seg[1] = up, out = seg[0].y
  QmvSeg seg[4];
  uint32_t items;       // output rows in total (pair: rows of the gate)
  int xmode;
  const float* x;       // input vector [cols]
  const float* xw;      // norm weight (XM_RMS1P: [cols], XM_GATED: [head_dim])
  const float* xaux;    // XM_GATED: z [cols]; XM_SIGGATE: gate [cols]
  float eps;
  uint32_t head_dim;    // XM_GATED
  int* err;             // device error word
  PeerOut peer;         // n > 0: sharded output (tensor-core Q4_K kernel only)
  void* scratch;        // the context's split-group scratch (zeroed counters first), may be null
  uint64_t scratch_bytes;
};

// Enqueue one launch. Returns SI_OK or SI_E_* with *msg filled.
int launch_qmv(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl,
               std::string* msg);

// Q6_K matvec on the tensor cores (qmatvec_tc6.cu): eligibility and launch;
// launch_qmv routes eligible Q6_K calls there.
// Measured on B200: the CUDA-core kernel stays ahead only on short matrices
// (1,024 rows of 20 or 48 blocks), so the tensor cores take 2,048 rows and
// more, or rows of 64 blocks and more (256 rows at least).
constexpr uint32_t kTc6MinRows = 256, kTc6AnyWidthRows = 2048, kTc6WideBlocks = 64;
constexpr uint64_t kQmvScratchBytes = 2ull << 20;  // one stream's split-group scratch
constexpr int kQmvScratchSlots = 8;                // streams per context with their own scratch
bool qmv_tc6_eligible(const QmvParams& p);
uint64_t qmv_tc6_scratch_bytes(uint32_t sm_count);  // the scratch a launch's split needs
int launch_qmv_tc6(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl, std::string* msg);

// Plain Q4_K matvec on the tensor cores (qmatvec_tc.cu): eligibility and
// launch; launch_qmv routes eligible calls there.
bool qmv_tc_eligible(const QmvParams& p);
// The tensor-core kernel on any row count (the sharded matvec with peer output).
bool qmv_tc_supported(const QmvParams& p);
int launch_qmv_tc(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl, std::string* msg);

// Batched matvec Y[k] = W X[k] (+ R[k]) for k < batch, one weight traversal.
constexpr uint32_t kQmmMaxBatch = 8;
struct QmmParams {
  uint32_t type, rows, cols, batch;
  const uint8_t* w;
  const float* x;       // x[k * ldx + c], 16-byte aligned, ldx % 4 == 0
  float* y;             // y[k * ldy + r]
  const float* resid;   // optional: y = resid + W x, resid[k * ldr + r] (may alias y)
  uint64_t ldx, ldy, ldr;
  void* scratch;        // device scratch for the tensor-core form (256-byte aligned), may be null
  uint64_t scratch_bytes;
  int* err;
  void* qscratch;       // the context's matvec scratch (batch 1 goes to the matvec family)
  uint64_t qscratch_bytes;
};
int launch_qmm(const QmmParams& p, cudaStream_t stream, int sm_count, bool pdl, std::string* msg);
// Tensor-core form for Q4_K (qmatmul_many_tc.cu): scratch it needs, whether a
// call qualifies, and the launch (SI_E_UNSUPPORTED: use the CUDA-core form).
uint64_t qmm_tc_scratch_bytes(uint32_t rows, uint32_t cols, uint32_t batch, int sm_count);
bool qmm_tc_eligible(const QmmParams& p);
int launch_qmm_tc(const QmmParams& p, cudaStream_t stream, int sm_count, bool pdl, std::string* msg);

// Largest supported column count (x and its partial sums live in shared memory).
constexpr uint32_t kQmvMaxCols = 32768;

}  // namespace si
