// Internal (C++) interfaces between the kernel files and the C ABI in capi.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace qg {

// Shared-memory budget for the staged activation tile of the GEMV kernels.
// A whole x of K <= 16384 floats (or N*K floats up to this size) is staged
// once per CTA; larger batches are staged in K tiles.
constexpr size_t kXStageBytes = 64 * 1024;

struct DeviceInfo {
  int device = 0;
  int sms = 0;
  int smem_optin = 0;  // max dynamic shared memory per block (opt-in)
  int cc_major = 0, cc_minor = 0;
  int l2_bytes = 0;
};

// Cached per device; fills `out` for the current device.
int current_device_info(DeviceInfo& out);

// Lets `func` use the device's opt-in shared-memory maximum (once per device).
int allow_max_smem(const void* func, const DeviceInfo& dev);

// Resident blocks per SM of `func` (cached per device, block size and smem).
int occupancy(const void* func, const DeviceInfo& dev, int threads, size_t smem, int* out);

// All-gather fused into the single-column GEMV (one process per GPU): the
// kernel also stores its rows into the other ranks' y buffers (peer
// pointers) and the CTA that finishes last adds 1 to every rank's counter
// sig_out[k]; with sig_in set, the kernel first waits (bounded) until the
// counter of its input reaches (*tok + 1) * nranks.
constexpr int kMaxRanks = 8;
struct FuseArgs {
  float* peer_y[kMaxRanks] = {};
  unsigned* sig_out[kMaxRanks] = {};
  unsigned* cta_count = nullptr;
  const unsigned* sig_in = nullptr;
  const unsigned* tok = nullptr;
  int npeer = 0, nranks = 0;
};

struct GemvCall {
  const void* q = nullptr;  // SoA quant plane, or AoS blocks
  const void* d = nullptr;  // SoA scale plane (fp16 bits); unused for AoS
  const float* x = nullptr;
  float* y = nullptr;
  int64_t M = 0, K = 0;
  int N = 1;
  int64_t ldx = 0, ldy = 0;
  int grid_override = 0;  // >0: force the grid size (tuning / tests)
  void* ws = nullptr;     // workspace of the tensor-core batch kernel
  size_t ws_bytes = 0;
  FuseArgs f;             // fused all-gather (f.nranks == 0: none)
  int act = 0;            // activations: 0 exact (fixed-point planes), 1 q8_1 (opt-in)
  bool no_tc = false;     // batched SoA: keep to the mma.sync kernel (fixed workspace)
};

int gemv_soa(int fmt, const GemvCall& c, cudaStream_t st);
int gemv_soa_variant(int fmt, int variant, const GemvCall& c, cudaStream_t st);
// TMA-fed single-column kernel; returns -1 when the shape is not eligible.
int gemv_soa_tma(int fmt, const GemvCall& c, cudaStream_t st);
bool tma_eligible(const GemvCall& c);
// mode 0: fp32 unpack + FFMA2; mode 1: fixed-point x planes + dp4a.
int gemv_soa_tma_mode(int fmt, int mode, const GemvCall& c, cudaStream_t st);
// GGUF-layout blocks on the TMA path; -1 when the shape is not eligible.
int gemv_aos_tma(int fmt, const GemvCall& c, cudaStream_t st);
// Two columns (N == 2) on the TMA path in one launch, SoA planes or GGUF
// blocks (exact activations; x columns 16-byte aligned); -1 when the call is
// not taken (tma_pair_taken: q4_0 planes and GGUF blocks).  Needs no
// workspace.
bool tma_pair_eligible(const GemvCall& c);
bool tma_pair_taken(int fmt, bool aos, const GemvCall& c);
int gemv_tma_pair(int fmt, bool aos, const GemvCall& c, cudaStream_t st);
int read_device_error(int clear, cudaStream_t st, int* out);
// Persistent decode stack: a sequence of single-column SoA GEMVs in one
// cooperative launch (GEMV j reads GEMV j-1's output).  Outputs are 8-byte
// slots (fp32 bits | tag << 32).  With P ranks (one GPU each) every GEMV's
// rows are also stored into the other ranks' slots (peer_y, rank order
// without this rank).
struct StackCall {
  const void* q;
  const void* d;
  const float* x;           // GEMV 0's input floats
  unsigned long long* y;    // this GEMV's output slots on this rank (M_total)
  int64_t r0, M, M_total, K;
  unsigned long long* peer_y[kMaxRanks - 1] = {};
};
struct StackRanks {
  int nranks = 1, rank = 0;
};
int stack_create(int fmt, const StackCall* calls, int n, const StackRanks* ranks, void** out);
int stack_run(void* handle, cudaStream_t st);
int stack_reset(void* handle, cudaStream_t st);
int stack_destroy(void* handle);
// End of a token of fused calls: signal every rank's done[k], wait (bounded)
// until done_local reaches (*tok + 1) * nranks, then advance *tok.
int token_fence(unsigned* const* done, int nranks, const unsigned* done_local, unsigned* tok,
                cudaStream_t st);
// Tensor-core kernel for 2..16 columns (needs c.ws); -1 when not eligible.
int gemv_soa_mma(int fmt, const GemvCall& c, cudaStream_t st);
bool mma_eligible(const GemvCall& c);
size_t mma_workspace_bytes(int64_t K, int N);
int read_mma_error(int clear, cudaStream_t st, int* out);
// Limits (clock64 cycles) of the bounded waits in the kernels of gemv_tma.cu
// and gemv_mma.cu, on the current device.
int set_spin_limit(long long cycles);
int set_mma_spin_limit(long long cycles);
constexpr long long kDefaultSpinLimit = 2000000000LL;  // ~1 s at ~2 GHz
// Tile counters handed out on `device` so far (one per stream that launched,
// one per captured launch; never returned) and the pool's size.
int tile_counters_used(int device);
int tile_counters_capacity();
// Batch tiles: the weights re-laid for the tensor-core kernel (one contiguous
// block per 16 rows x 512 columns); any K % 32 == 0.
size_t tiled_bytes(int fmt, int64_t M, int64_t K);
int tile_weights(int fmt, bool aos, const void* q, const void* d, int64_t M, int64_t K,
                 void* out, cudaStream_t st);
int gemv_tiled(int fmt, const GemvCall& c, cudaStream_t st);  // c.q = tiles, 1..16 columns
// tc tiles and the tcgen05 batch kernel (gemv_tc.cu), q8_0 (fmt 8) and q4_0
// (fmt 4): 1..16 columns per call; the workspace bound holds for every column
// count and both formats on a device with `sms` SMs.
size_t tc_tiles_bytes(int fmt, int64_t M, int64_t K);
size_t tc_workspace_bytes(int64_t M, int64_t K, int sms);
int tile_weights_tc(int fmt, bool aos, const void* q, const void* d, int64_t M, int64_t K,
                    void* out, cudaStream_t st);
int gemv_tc(int fmt, const void* tiles, int64_t M, int64_t K, const float* x, int64_t ldx,
            float* y, int64_t ldy, int N, void* ws, size_t ws_bytes, cudaStream_t st);
// The same kernel streaming SoA planes through 2-D tensor copies (no
// re-layout): K % 256 == 0, q and d 16-byte aligned; -1 when not eligible or
// when c.ws_bytes is below tc_soa_workspace_bytes.
int gemv_soa_tc(int fmt, const GemvCall& c, cudaStream_t st);
size_t tc_soa_workspace_bytes(int64_t M, int64_t K, int N, int sms);
// A 2-D tensor map (uint8 or uint16 elements; inner dimension contiguous).
int encode_tensor_2d(CUtensorMap* map, bool u16, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
int set_tc_spin_limit(long long cycles);
int read_tc_error(int clear, cudaStream_t st, int* out);
// Workspace cached per (device, stream) for callers that pass none; grows on
// demand (cudaMalloc, outside stream capture only).
int stream_workspace(cudaStream_t st, size_t bytes, void** out);
// The fixed per-device workspace of qgemv_soa_static_ws (static_ws.cu).
constexpr size_t kStaticWsBytes = (size_t)2 << 20;
int static_workspace(void** out, size_t* bytes);
int release_workspaces();
int soa_variant_count();
const char* soa_variant_name(int v);
int gemv_aos(int fmt, const GemvCall& c, cudaStream_t st);
int fill_zero_rows(float* y, int64_t M, int N, int64_t ldy, cudaStream_t st);

// Quantizers: W fp32 [M][ldw] -> SoA planes (q, d) or AoS blocks.
int quantize(int fmt, const float* w, int64_t M, int64_t K, int64_t ldw, void* q, void* d,
             void* aos, cudaStream_t st);
int dequant(int fmt, const void* q, const void* d, float* w, int64_t M, int64_t K,
            cudaStream_t st);
int repack(int fmt, int to_soa, const void* aos, void* q, void* d, int64_t M, int64_t K,
           cudaStream_t st);

// Roof probes.
int roof_stream_read(const void* buf, size_t bytes, uint32_t* sink, int blocks_per_sm,
                     cudaStream_t st);
int roof_bulk_read(const void* buf, size_t bytes, uint32_t* sink, int* status,
                   cudaStream_t st);

}  // namespace qg
