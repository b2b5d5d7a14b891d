// AlphaZero ResNet policy/value forward on B200 (reference: ResNetModel.forward,
// python/mcts/neural_networks/resnet_model.py:247-271, evaluated as in
// ResNetEvaluator._forward_model, resnet_evaluator.py:231-265 -> policy = exp(log_softmax)).
//
// Trunk: every 3x3 convolution (BN folded into weight + bias) is one persistent implicit-GEMM
// kernel on the 5th-generation tensor cores, k_conv3x3_halo_t, in transposed form:
//   M = 128 output channels (from the weights), N = 256 pixels, K = 9 taps x input channels;
// with 256 filters every 256-pixel tile is two work items, one per half of the output channels.
// Activations live in a padded pixel space: each position is a (S+1) x (S+1) grid whose last
// row and last column are zero (S = board size). Flattened row-major, the grid makes every 3x3
// tap a constant row shift (dy*(S+1) + dx) of the same matrix - the zero column serves as both
// the left and the right border, and the zero row of position b as the top border of b+1 - so
// one TMA load per 64-channel block brings a tile's pixels plus a halo of rows on each side into
// shared memory, and each tap's UMMA reads a row-shifted window of it (rows before the tensor
// start read as zeros).
// Warp roles per CTA: warp 0 TMA producer, warp 1 MMA issuer (single thread, tcgen05.mma with
// both operands in 128B-swizzled shared memory), warps 2-13 epilogue (TMEM -> registers, + bias,
// + residual, ReLU, zero the pad pixels, 16-bit TMA store). Accumulators are double-buffered in
// TMEM so the epilogue of one tile overlaps the MMAs of the next.
// Heads: 1x1 convolutions into 16-bit rows, then the fully connected layers on the tensor cores
// (k_dense) with fused bias/ReLU, softmax or value dot + tanh; SIMT k_heads where the widths do
// not fit the dense tiles and in the no-allocation entry point.
#include <cuda.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <new>

#include "omq_internal.cuh"
#include "sm100_ptx.cuh"

namespace omq {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait before giving up
constexpr int kBlockK = 64;     // 64 bf16 = one 128-byte swizzle row
constexpr int kInPad = 64;      // input planes padded to one K block (two for more than 64 planes)
__host__ __device__ constexpr int in_pad_of(int planes) { return planes <= kInPad ? kInPad : 2 * kInPad; }
constexpr int kMaxInputPlanes = 2 * kInPad;
constexpr int kMaxActions = 5000;

struct ConvArgs {
  const float* bias;
  const h16* residual;
  h16* out;
  const int32_t* d_count;
  int32_t count;
  int32_t P;
  int32_t S;
  int32_t kb_per_tap;
  int32_t relu;
  int32_t* error;
  int32_t halves;  // transposed halo kernel: output channels / 128 (each work item is one half)
};

// Pipeline of the transposed halo kernel: 4 weight stages, 12 epilogue warps with one TMA-store
// buffer each. With 128 filters the epilogue (transpose, bias, residual, store) of a 256-pixel tile
// has only 72 UMMAs of MMA time to hide behind: 12 epilogue warps ran ResNet 10x128 1-3% faster
// than 8 (config 1 +1.5% at a 3% lower SM clock), 4 warps 15% slower; 256 filters were unchanged.
constexpr int kHaloWStages = 4, kHaloEpiWarps = 12, kHaloStoreBufs = 1;

// Transposed halo kernel (128 and 256 filters): D[channel][pixel] = W[channel][K] . X[pixel][K]^T, so
// each UMMA is M = 128 output channels x N = 256 pixels x K = 16. The pixel operand is the same
// row-shifted window of the halo buffer as in k_conv3x3_halo (one 304-row TMA load per 64-channel
// block). A 128 x 256 x 16 UMMA keeps the tensor pipe busy for 128 cycles, twice as long as a
// 128 x 128 x 16 one, which leaves the single issuing thread enough time for its barrier waits and
// commits (measured on B200: with 128 x 128 x 16 UMMAs any per-step work of the issuer idles the
// tensor pipe; with 128 x 256 x 16 none does). The epilogue receives channel-major accumulators
// (TMEM lane = channel) and transposes them through a swizzled fp32 buffer per warp, so that each
// lane then owns one pixel row: residual loads, padding and the TMA-store staging stay row-major.
template <int WS, int EW, int SB>
struct HaloTCfgT {
  static constexpr int kRows = 256;                          // pixels per tile (UMMA N)
  static constexpr int kLead = 24;                           // halo rows before the tile (>= S+2)
  static constexpr int kHaloRows = 304;
  static constexpr int kHaloBox = 152;
  static constexpr int kX = kHaloRows * 128;                 // one 64-channel halo block, 38,912 B
  static constexpr int kXStages = 2;
  static constexpr int kW = 128 * 128;                       // one tap's weights (128 ch x 64 K), 16 KB
  static constexpr int kWStages = WS;                          // weight stages in flight
  static constexpr int kEpiWarps = EW;                         // a multiple of 4 (TMEM lane quarters)
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kTmemCols = 512;                      // 2 buffers x 256 pixel columns
  static constexpr int kStoreBufs = SB;                      // 16-bit TMA-store buffers per epilogue warp
  static constexpr int kStagePerWarp = SB * 2048 + 4096;     // store buffers + fp32 transpose
  static constexpr int kStaging = kEpiWarps * kStagePerWarp;
  static constexpr int kSmem = kXStages * kX + kWStages * kW + kStaging + 1024 + 512 + 256 * 4;
  static_assert(kSmem <= 232448, "227 KB of shared memory per CTA");
  static_assert(EW % 4 == 0, "epilogue warps cover the 4 TMEM lane quarters");
};
using HaloTCfg = HaloTCfgT<kHaloWStages, kHaloEpiWarps, kHaloStoreBufs>;

template <bool F16>
__global__ void __launch_bounds__(HaloTCfg::kThreads, 1)
    k_conv3x3_halo_t(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO, ConvArgs args) {
  using Cfg = HaloTCfg;
  constexpr int BN = 128;  // output channels of one work item (one half of 256 filters)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* x_ring = smem;                                     // 2 x 38,912
  uint8_t* w_ring = smem + Cfg::kXStages * Cfg::kX;           // 4 x 16 KB
  uint8_t* staging = w_ring + Cfg::kWStages * Cfg::kW;
  uint64_t* xfull = reinterpret_cast<uint64_t*>(staging + Cfg::kStaging);
  uint64_t* xempty = xfull + Cfg::kXStages;
  uint64_t* wfull = xempty + Cfg::kXStages;
  uint64_t* wempty = wfull + Cfg::kWStages;
  uint64_t* tfull = wempty + Cfg::kWStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_bias = reinterpret_cast<float*>(staging + Cfg::kStaging + 512);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // work item w: pixel tile w / halves, output channels [128 * (w % halves), +128)
  const int halves = args.halves;
  const int cout = BN * halves;
  const int CB = args.kb_per_tap;
  const int rowstride = args.S + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kXStages; ++s) { ptx::mbar_init(&xfull[s], 1); ptx::mbar_init(&xempty[s], 1); }
    for (int s = 0; s < Cfg::kWStages; ++s) { ptx::mbar_init(&wfull[s], 1); ptx::mbar_init(&wempty[s], 1); }
    for (int i = 0; i < 2; ++i) { ptx::mbar_init(&tfull[i], 1); ptx::mbar_init(&tempty[i], Cfg::kEpiWarps); }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tmap(&tmH);
    ptx::prefetch_tmap(&tmB);
    ptx::prefetch_tmap(&tmO);
  }
  for (int i = threadIdx.x; i < cout; i += blockDim.x) s_bias[i] = args.bias[i];
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, Cfg::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched as a programmatic dependent of the previous kernel in the stream, the setup above
  // (barriers, TMEM, tensor-map prefetch, bias) overlaps that kernel's tail; every global read
  // of its outputs and every global write comes after this wait for its completion.
  ptx::griddep_wait();
  const int n_pos = args.d_count ? min(*args.d_count, args.count) : args.count;
  const int rows = n_pos * args.P;
  const int tiles = (rows + Cfg::kRows - 1) / Cfg::kRows;
  const int items = tiles * halves;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: per 64-channel block one halo, then 9 weight taps -------
    int sx = 0, sw = 0;
    uint32_t px = 0, pw = 0;
    int x_issued[Cfg::kXStages], w_issued[Cfg::kWStages];
    for (int i = 0; i < Cfg::kXStages; ++i) x_issued[i] = -1;
    for (int i = 0; i < Cfg::kWStages; ++i) w_issued[i] = -1;
    for (int w = blockIdx.x; w < items && !*abort_flag; w += gridDim.x) {
      const int tile = w / halves, half = w - tile * halves;
      const int h0 = tile * Cfg::kRows - Cfg::kLead;
      for (int cb = 0; cb < CB; ++cb) {
        if (!ptx::mbar_wait(&xempty[sx], px ^ 1, abort_flag, kWaitLimitNs)) goto producer_done;
        ptx::mbar_arrive_expect_tx(&xfull[sx], Cfg::kX);
        uint8_t* dst = x_ring + sx * Cfg::kX;
        ptx::tma_load_2d(dst, &tmH, &xfull[sx], cb * kBlockK, h0);
        ptx::tma_load_2d(dst + Cfg::kHaloBox * 128, &tmH, &xfull[sx], cb * kBlockK, h0 + Cfg::kHaloBox);
        x_issued[sx] = (int)px;
        if (++sx == Cfg::kXStages) { sx = 0; px ^= 1; }
        for (int tap = 0; tap < 9; ++tap) {
          if (!ptx::mbar_wait(&wempty[sw], pw ^ 1, abort_flag, kWaitLimitNs)) goto producer_done;
          ptx::mbar_arrive_expect_tx(&wfull[sw], Cfg::kW);
          ptx::tma_load_2d(w_ring + sw * Cfg::kW, &tmB, &wfull[sw], (tap * CB + cb) * kBlockK, half * BN);
          w_issued[sw] = (int)pw;
          if (++sw == Cfg::kWStages) { sw = 0; pw ^= 1; }
        }
      }
    }
  producer_done:
    for (int i = 0; i < Cfg::kXStages; ++i)
      if (x_issued[i] >= 0) {
        volatile int dummy = 0;
        ptx::mbar_wait(&xfull[i], (uint32_t)x_issued[i], &dummy, kWaitLimitNs);
      }
    for (int i = 0; i < Cfg::kWStages; ++i)
      if (w_issued[i] >= 0) {
        volatile int dummy = 0;
        ptx::mbar_wait(&wfull[i], (uint32_t)w_issued[i], &dummy, kWaitLimitNs);
      }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer: A = weights (M = 128 channels), B = pixel window (N = 256) ----
    // When a tile is exactly one position (P = 256: the 16x16 grid of a 15x15 board) its last grid
    // row is the zero pad row: no real output reads past pixel 255 of the tile (largest tap shift
    // S + 2 from pixel 14*16 + 14), and the pad row's outputs are written as zeros by the
    // epilogue, so the UMMAs cover only the first 256 - 16 = 240 pixel columns.
    const uint32_t idesc =
        ptx::idesc_f16_f32(BN, args.P == Cfg::kRows ? Cfg::kRows - rowstride : Cfg::kRows, F16);
    const uint64_t w_desc0 = ptx::smem_desc_sw128(ptx::smem_u32(w_ring));
    int sx = 0, sw = 0;
    uint32_t px = 0, pw = 0;
    bool any = false;
    int t = 0;
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++t) {
      const int ab = t & 1;
      const uint32_t aph = (t >> 1) & 1;
      if (!ptx::mbar_wait(&tempty[ab], aph ^ 1, abort_flag, kWaitLimitNs)) break;
      ptx::tc_fence_after();
      const uint32_t d = tmem + ab * Cfg::kRows;
      bool ok = true;
      for (int cb = 0; cb < CB && ok; ++cb) {
        if (!ptx::mbar_wait(&xfull[sx], px, abort_flag, kWaitLimitNs)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint64_t x_desc0 = ptx::smem_desc_sw128(ptx::smem_u32(x_ring + sx * Cfg::kX));
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          if (!ptx::mbar_wait(&wfull[sw], pw, abort_flag, kWaitLimitNs)) { ok = false; break; }
          ptx::tc_fence_after();
          const int off = Cfg::kLead + (tap / 3 - 1) * rowstride + (tap % 3 - 1);
          const uint64_t xd = x_desc0 + (uint64_t)(off * 8);             // off rows of 128 B
          const uint64_t wd = w_desc0 + (uint64_t)(sw * (Cfg::kW >> 4));
          ptx::mma_f16(d, wd, xd, idesc, (cb | tap) != 0);
#pragma unroll
          for (int k = 1; k < kBlockK / 16; ++k) ptx::mma_f16(d, wd + 2 * k, xd + 2 * k, idesc, 1u);
          any = true;
          ptx::mma_commit(&wempty[sw]);
          if (++sw == Cfg::kWStages) { sw = 0; pw ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit(&xempty[sx]);
        if (++sx == Cfg::kXStages) { sx = 0; px ^= 1; }
      }
      if (!ok) break;
      ptx::mma_commit(&tfull[ab]);
    }
    if (any) {
      ptx::mma_commit(drain);
      volatile int dummy = 0;
      ptx::mbar_wait(drain, 0, &dummy, kWaitLimitNs);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    // Warp w reads TMEM lanes (= output channels) 32q..32q+31, q = w % 4; the two warps of a lane
    // quarter take alternate 32-pixel column chunks of the tile.
    const int q = warp & 3;
    const int wq = (warp - 2) >> 2;
    uint8_t* my_stage = staging + (warp - 2) * Cfg::kStagePerWarp;
    float* tr = reinterpret_cast<float*>(my_stage + Cfg::kStoreBufs * 2048);  // [32 px][32 ch] fp32, swizzled
    int buf = 0;
    int t = 0;
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++t) {
      const int tile = w / halves, half = w - tile * halves;
      const int ch0 = half * BN + q * 32;  // this warp's first output channel
      const float bias = s_bias[ch0 + lane];
      const int ab = t & 1;
      const uint32_t aph = (t >> 1) & 1;
      if (!ptx::mbar_wait(&tfull[ab], aph, abort_flag, kWaitLimitNs)) break;
      ptx::tc_fence_after();
#pragma unroll 1
      for (int j = wq; j < Cfg::kRows / 32; j += Cfg::kEpiWarps / 4) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + ab * Cfg::kRows + j * 32, r);
        ptx::tmem_ld_wait();
        // transpose: this lane holds channel c = lane for pixels 0..31 of the chunk; word (p, c)
        // lives at p * 32 + ((c / 4) ^ (p % 8)) * 4 + c % 4 (conflict-free both ways)
        __syncwarp();
#pragma unroll
        for (int p = 0; p < 32; ++p)
          tr[p * 32 + (((lane >> 2) ^ (p & 7)) << 2) + (lane & 3)] = __uint_as_float(r[p]) + bias;
        __syncwarp();
        const int row0 = tile * Cfg::kRows + j * 32;
        const int m = row0 + lane;
        const bool valid = m < rows;
        const int pix = m % args.P;
        const int y = pix / rowstride, x = pix - y * rowstride;
        const bool pad = !valid || (y == args.S) || (x == args.S);
        uint4 packed[4];
        uint32_t* pwd = reinterpret_cast<uint32_t*>(packed);
        if (pad) {
#pragma unroll
          for (int i = 0; i < 16; ++i) pwd[i] = 0u;
        } else {
          float v[32];
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            const float4 f = *reinterpret_cast<const float4*>(tr + lane * 32 + ((c4 ^ (lane & 7)) << 2));
            v[4 * c4] = f.x; v[4 * c4 + 1] = f.y; v[4 * c4 + 2] = f.z; v[4 * c4 + 3] = f.w;
          }
          if (args.residual) {
            const uint4* rp = reinterpret_cast<const uint4*>(args.residual + (size_t)m * cout + ch0);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint4 u = rp[i];
              const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack2_h16<F16>(uw[e]);
                v[8 * i + 2 * e] += f.x;
                v[8 * i + 2 * e + 1] += f.y;
              }
            }
          }
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float v0 = v[i], v1 = v[i + 1];
            if (args.relu) { v0 = fmaxf(v0, 0.0f); v1 = fmaxf(v1, 0.0f); }
            pwd[i / 2] = pack2_h16<F16>(v0, v1);
          }
        }
        // the buffer about to be written must no longer be read by an earlier store
        if (lane == 0) ptx::bulk_wait_read<Cfg::kStoreBufs - 1>();
        __syncwarp();
        uint8_t* sbuf = my_stage + buf * 2048;
        const int swz = (lane >> 1) & 3;
#pragma unroll
        for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(sbuf + lane * 64 + ((i ^ swz) * 16)) = packed[i];
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::tma_store_2d(&tmO, sbuf, ch0, row0);
          ptx::bulk_commit();
        }
        if (++buf == Cfg::kStoreBufs) buf = 0;
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&tempty[ab]);
    }
    if (lane == 0) ptx::bulk_wait<0>();
  }
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(args.error, OMQ_TIMEOUT);
}

// ---------------------------------------------------------------------------------------------
// Whole trunk in one launch, for boards whose padded grid is exactly one 256-pixel tile (15x15)
// with 128 filters: a tile is a whole position, so every layer of a position depends only on the
// previous layer of the same position, and one CTA can run all 1 + 2 NB convs of its positions
// with no other CTA involved. Each CTA keeps two positions in flight in the two TMEM accumulators
// (items alternate position A layer l, position B layer l, A layer l+1, ...): while the MMAs of B
// run, the epilogue of A drains and stores, and A's next layer starts once those stores have
// completed (the per-slot `stored` barrier, which the TMA producer waits on before loading A's
// next halo). The layers' activations live in a per-CTA scratch of 3 buffers x 2 slots (64 KB
// per buffer and slot, L2-resident and rewritten in place) instead of three full-batch buffers:
// only the input features and the trunk's output cross DRAM. Same MMAs, same epilogue arithmetic
// and the same K order as the layer-by-layer kernel, so the results are identical to it.
// ---------------------------------------------------------------------------------------------
struct TrunkArgs {
  const float* bias;       // [1 + 2 NB][128]
  const h16* scratch;      // [3][nslots][256][128] (residual reads; writes go through tmSo)
  const int32_t* d_count;
  int32_t count;
  int32_t layers;          // 1 + 2 NB
  int32_t cb_in;           // 64-channel blocks of the input (1 or 2)
  int32_t nslots;          // 2 x gridDim.x
  int32_t* error;
};

// Scratch buffer (0..2) read by layer l >= 1 as its input, or as its residual (conv2 layers), and
// written as its output. Block i = (l - 1) / 2 starts from buffer (2 i) % 3; conv1 writes the next
// buffer, conv2 the one after (the rotation of the layer-by-layer forward).
__device__ __forceinline__ int trunk_in_buf(int l) { const int x = (2 * ((l - 1) >> 1)) % 3; return (l & 1) ? x : (x + 1) % 3; }
__device__ __forceinline__ int trunk_out_buf(int l) {
  if (l == 0) return 0;
  const int x = (2 * ((l - 1) >> 1)) % 3;
  return (l & 1) ? (x + 1) % 3 : (x + 2) % 3;
}
__device__ __forceinline__ int trunk_res_buf(int l) { return (2 * ((l - 1) >> 1)) % 3; }

template <bool F16>
__global__ void __launch_bounds__(HaloTCfg::kThreads, 1)
    k_trunk_t(const __grid_constant__ CUtensorMap tmIn, const __grid_constant__ CUtensorMap tmWin,
              const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
              const __grid_constant__ CUtensorMap tmSo, const __grid_constant__ CUtensorMap tmOut,
              TrunkArgs args) {
  using Cfg = HaloTCfg;
  constexpr int C = 128, kP = 256, kStride = 16, kN = kP - kStride;  // 240 pixel columns per UMMA
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* x_ring = smem;
  uint8_t* w_ring = smem + Cfg::kXStages * Cfg::kX;
  uint8_t* staging = w_ring + Cfg::kWStages * Cfg::kW;
  uint64_t* xfull = reinterpret_cast<uint64_t*>(staging + Cfg::kStaging);
  uint64_t* xempty = xfull + Cfg::kXStages;
  uint64_t* wfull = xempty + Cfg::kXStages;
  uint64_t* wempty = wfull + Cfg::kWStages;
  uint64_t* tfull = wempty + Cfg::kWStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* stored = tempty + 2;  // [2] per slot: the item's output stores have completed
  uint64_t* drain = stored + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kXStages; ++s) { ptx::mbar_init(&xfull[s], 1); ptx::mbar_init(&xempty[s], 1); }
    for (int s = 0; s < Cfg::kWStages; ++s) { ptx::mbar_init(&wfull[s], 1); ptx::mbar_init(&wempty[s], 1); }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&tfull[i], 1);
      ptx::mbar_init(&tempty[i], Cfg::kEpiWarps);
      ptx::mbar_init(&stored[i], Cfg::kEpiWarps);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tmap(&tmIn);
    ptx::prefetch_tmap(&tmWin);
    ptx::prefetch_tmap(&tmW);
    ptx::prefetch_tmap(&tmS);
    ptx::prefetch_tmap(&tmSo);
    ptx::prefetch_tmap(&tmOut);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, Cfg::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  ptx::griddep_wait();
  const int n_pos = args.d_count ? min(*args.d_count, args.count) : args.count;
  // this CTA's positions: blockIdx.x + k * gridDim.x, k = 0 .. mine - 1, in pairs (2m, 2m + 1)
  const int mine = n_pos > (int)blockIdx.x ? (n_pos - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int L = args.layers;
  // the item sequence every role walks: pair m, layer l, position k = 2m + j of the pair
#define OMQ_TRUNK_ITEMS(...)                                            \
  for (int m = 0; 2 * m < mine; ++m)                                    \
    for (int l = 0; l < L; ++l)                                         \
      for (int j = 0; j < 2 && 2 * m + j < mine; ++j) {                 \
        const int k = 2 * m + j;                                        \
        const int pos = (int)blockIdx.x + k * (int)gridDim.x;           \
        const int sl = j, slot = 2 * (int)blockIdx.x + j;               \
        __VA_ARGS__                                                     \
      }

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int sx = 0, sw = 0;
    uint32_t px = 0, pw = 0;
    int x_issued[Cfg::kXStages], w_issued[Cfg::kWStages];
    for (int i = 0; i < Cfg::kXStages; ++i) x_issued[i] = -1;
    for (int i = 0; i < Cfg::kWStages; ++i) w_issued[i] = -1;
    int done_items[2] = {0, 0};  // items of each slot issued so far
    bool ok = true;
    const uint64_t pol_last = ptx::l2_policy_evict_last(), pol_first = ptx::l2_policy_evict_first();
    OMQ_TRUNK_ITEMS({
      if (ok) {
        // the previous item of this slot (its previous layer, or the previous position's last
        // one) must have stored its output before this item's input loads or output stores
        if (done_items[sl] > 0) {
          if (!ptx::mbar_wait(&stored[sl], (uint32_t)((done_items[sl] - 1) & 1), abort_flag, kWaitLimitNs)) ok = false;
          ptx::fence_proxy_async_global();
        }
        ++done_items[sl];
        const int CB = l == 0 ? args.cb_in : C / kBlockK;
        const int h0 = l == 0 ? pos * kP - Cfg::kLead : (trunk_in_buf(l) * args.nslots + slot) * kP - Cfg::kLead;
        const CUtensorMap* hm = l == 0 ? &tmIn : &tmS;
        const CUtensorMap* wm = l == 0 ? &tmWin : &tmW;
        const int wrow = l == 0 ? 0 : (l - 1) * C;
        // scratch lines are rewritten by the next positions: keep them in L2; the input features
        // are read once
        const uint64_t pol = l == 0 ? pol_first : pol_last;
        for (int cb = 0; cb < CB && ok; ++cb) {
          if (!ptx::mbar_wait(&xempty[sx], px ^ 1, abort_flag, kWaitLimitNs)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(&xfull[sx], Cfg::kX);
          uint8_t* dst = x_ring + sx * Cfg::kX;
          ptx::tma_load_2d_hint(dst, hm, &xfull[sx], cb * kBlockK, h0, pol);
          ptx::tma_load_2d_hint(dst + Cfg::kHaloBox * 128, hm, &xfull[sx], cb * kBlockK, h0 + Cfg::kHaloBox, pol);
          x_issued[sx] = (int)px;
          if (++sx == Cfg::kXStages) { sx = 0; px ^= 1; }
          for (int tap = 0; tap < 9; ++tap) {
            if (!ptx::mbar_wait(&wempty[sw], pw ^ 1, abort_flag, kWaitLimitNs)) { ok = false; break; }
            ptx::mbar_arrive_expect_tx(&wfull[sw], Cfg::kW);
            ptx::tma_load_2d(w_ring + sw * Cfg::kW, wm, &wfull[sw], (tap * CB + cb) * kBlockK, wrow);
            w_issued[sw] = (int)pw;
            if (++sw == Cfg::kWStages) { sw = 0; pw ^= 1; }
          }
        }
      }
    })
    for (int i = 0; i < Cfg::kXStages; ++i)
      if (x_issued[i] >= 0) {
        volatile int dummy = 0;
        ptx::mbar_wait(&xfull[i], (uint32_t)x_issued[i], &dummy, kWaitLimitNs);
      }
    for (int i = 0; i < Cfg::kWStages; ++i)
      if (w_issued[i] >= 0) {
        volatile int dummy = 0;
        ptx::mbar_wait(&wfull[i], (uint32_t)w_issued[i], &dummy, kWaitLimitNs);
      }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = ptx::idesc_f16_f32(C, kN, F16);
    const uint64_t w_desc0 = ptx::smem_desc_sw128(ptx::smem_u32(w_ring));
    int sx = 0, sw = 0;
    uint32_t px = 0, pw = 0;
    bool any = false, ok = true;
    int t = 0;
    OMQ_TRUNK_ITEMS({
      if (ok) {
        (void)pos; (void)sl; (void)slot;
        const int ab = t & 1;
        const uint32_t aph = (t >> 1) & 1;
        ++t;
        if (!ptx::mbar_wait(&tempty[ab], aph ^ 1, abort_flag, kWaitLimitNs)) ok = false;
        ptx::tc_fence_after();
        const uint32_t d = tmem + ab * Cfg::kRows;
        const int CB = l == 0 ? args.cb_in : C / kBlockK;
        for (int cb = 0; cb < CB && ok; ++cb) {
          if (!ptx::mbar_wait(&xfull[sx], px, abort_flag, kWaitLimitNs)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint64_t x_desc0 = ptx::smem_desc_sw128(ptx::smem_u32(x_ring + sx * Cfg::kX));
#pragma unroll
          for (int tap = 0; tap < 9; ++tap) {
            if (!ptx::mbar_wait(&wfull[sw], pw, abort_flag, kWaitLimitNs)) { ok = false; break; }
            ptx::tc_fence_after();
            const int off = Cfg::kLead + (tap / 3 - 1) * kStride + (tap % 3 - 1);
            const uint64_t xd = x_desc0 + (uint64_t)(off * 8);
            const uint64_t wd = w_desc0 + (uint64_t)(sw * (Cfg::kW >> 4));
            ptx::mma_f16(d, wd, xd, idesc, (cb | tap) != 0);
#pragma unroll
            for (int kk = 1; kk < kBlockK / 16; ++kk) ptx::mma_f16(d, wd + 2 * kk, xd + 2 * kk, idesc, 1u);
            any = true;
            ptx::mma_commit(&wempty[sw]);
            if (++sw == Cfg::kWStages) { sw = 0; pw ^= 1; }
          }
          if (!ok) break;
          ptx::mma_commit(&xempty[sx]);
          if (++sx == Cfg::kXStages) { sx = 0; px ^= 1; }
        }
        if (ok) ptx::mma_commit(&tfull[ab]);
      }
    })
    if (any) {
      ptx::mma_commit(drain);
      volatile int dummy = 0;
      ptx::mbar_wait(drain, 0, &dummy, kWaitLimitNs);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue (as in k_conv3x3_halo_t) ----------------
    const int q = warp & 3;
    const int wq = (warp - 2) >> 2;
    uint8_t* my_stage = staging + (warp - 2) * Cfg::kStagePerWarp;
    float* tr = reinterpret_cast<float*>(my_stage + Cfg::kStoreBufs * 2048);
    int buf = 0, t = 0;
    bool ok = true;
    const uint64_t pol_last = ptx::l2_policy_evict_last(), pol_first = ptx::l2_policy_evict_first();
    OMQ_TRUNK_ITEMS({
      if (ok) {
        const int ch0 = q * 32;
        const float bias = args.bias[(size_t)l * C + ch0 + lane];
        const int ab = t & 1;
        const uint32_t aph = (t >> 1) & 1;
        ++t;
        if (!ptx::mbar_wait(&tfull[ab], aph, abort_flag, kWaitLimitNs)) ok = false;
        ptx::tc_fence_after();
        const bool last = l == L - 1;
        const CUtensorMap* om = last ? &tmOut : &tmSo;
        const int orow0 = last ? pos * kP : (trunk_out_buf(l) * args.nslots + slot) * kP;
        const h16* res = (l >= 2 && !(l & 1))
                             ? args.scratch + ((size_t)(trunk_res_buf(l) * args.nslots + slot) * kP) * C
                             : nullptr;
#pragma unroll 1
        for (int jj = wq; ok && jj < Cfg::kRows / 32; jj += Cfg::kEpiWarps / 4) {
          uint32_t r[32];
          ptx::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + ab * Cfg::kRows + jj * 32, r);
          ptx::tmem_ld_wait();
          __syncwarp();
#pragma unroll
          for (int pp = 0; pp < 32; ++pp)
            tr[pp * 32 + (((lane >> 2) ^ (pp & 7)) << 2) + (lane & 3)] = __uint_as_float(r[pp]) + bias;
          __syncwarp();
          const int pix = jj * 32 + lane;
          const int y = pix / kStride, x = pix - y * kStride;
          const bool pad = (y == kStride - 1) || (x == kStride - 1);
          uint4 packed[4];
          uint32_t* pwd = reinterpret_cast<uint32_t*>(packed);
          if (pad) {
#pragma unroll
            for (int i = 0; i < 16; ++i) pwd[i] = 0u;
          } else {
            float v[32];
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 f = *reinterpret_cast<const float4*>(tr + lane * 32 + ((c4 ^ (lane & 7)) << 2));
              v[4 * c4] = f.x; v[4 * c4 + 1] = f.y; v[4 * c4 + 2] = f.z; v[4 * c4 + 3] = f.w;
            }
            if (res) {
              // written by this CTA's TMA stores two items earlier: read from L2, never from a
              // possibly stale L1 line of an earlier position in the same slot
              const uint4* rp = reinterpret_cast<const uint4*>(res + (size_t)pix * C + ch0);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 u = __ldcg(rp + i);
                const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = unpack2_h16<F16>(uw[e]);
                  v[8 * i + 2 * e] += f.x;
                  v[8 * i + 2 * e + 1] += f.y;
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 32; i += 2) pwd[i / 2] = pack2_h16<F16>(fmaxf(v[i], 0.0f), fmaxf(v[i + 1], 0.0f));
          }
          if (lane == 0) ptx::bulk_wait_read<Cfg::kStoreBufs - 1>();
          __syncwarp();
          uint8_t* sbuf = my_stage + buf * 2048;
          const int swz = (lane >> 1) & 3;
#pragma unroll
          for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(sbuf + lane * 64 + ((i ^ swz) * 16)) = packed[i];
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d_hint(om, sbuf, ch0, orow0 + jj * 32, last ? pol_first : pol_last);
            ptx::bulk_commit();
          }
          if (++buf == Cfg::kStoreBufs) buf = 0;
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          ptx::mbar_arrive(&tempty[ab]);
          // the item's stores complete (written, not only read from shared memory) before the
          // producer may load them as the next layer's input
          ptx::bulk_wait<0>();
          ptx::fence_proxy_async_global();
          ptx::mbar_arrive(&stored[sl]);
        }
        __syncwarp();
      }
    })
    if (lane == 0) ptx::bulk_wait<0>();
  }
#undef OMQ_TRUNK_ITEMS
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(args.error, OMQ_TIMEOUT);
}

// ---------------------------------------------------------------------------------------------
// input packing: reference fp32 features [n][planes][S][S] -> bf16 or fp16 [n][P][in_pad] padded
// pixel space
// ---------------------------------------------------------------------------------------------
__global__ void k_pack_features(const float* feat, int planes, int S, int P, const int32_t* d_count,
                                int count, bool f16, h16* out) {
  const int n = d_count ? min(*d_count, count) : count;
  const int total = n * P;
  const int C = S * S;
  const int chunks = in_pad_of(planes) / 8;  // chunks of 8 channels per pixel
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total * chunks; i += gridDim.x * blockDim.x) {
    const int row = i / chunks, chunk = i - row * chunks;
    const int b = row / P, pix = row - b * P;
    const int y = pix / (S + 1), x = pix - y * (S + 1);
    uint4 u = make_uint4(0, 0, 0, 0);
    if (y < S && x < S) {
      h16 h[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = chunk * 8 + e;
        const float v = c < planes ? feat[((size_t)b * planes + c) * C + y * S + x] : 0.0f;
        h[e] = to_h16(v, f16);
      }
      u = *reinterpret_cast<uint4*>(h);
    }
    reinterpret_cast<uint4*>(out)[(size_t)row * chunks + chunk] = u;
  }
}


// ---------------------------------------------------------------------------------------------
// heads on the tensor cores: 1x1 convolutions into bf16 rows, then one tcgen05 dense layer per
// fully connected layer (M = 128 positions x N <= 256 outputs per UMMA, bf16 in, fp32 accumulate)
// with the layer's epilogue fused (bias + ReLU -> bf16, softmax, or the value dot + tanh).
// ---------------------------------------------------------------------------------------------
enum DenseMode { kDenseRelu16 = 0, kDenseSoftmax = 1, kDenseLogits = 2, kDenseValue = 3 };

struct DenseArgs {
  const float* bias;       // [n_total]
  const float* w2;         // value mode: fc2 weights [n_total]
  const float* b2;         // value mode: fc2 bias [1]
  void* out;               // 16-bit [rows][ld] | fp32 [rows][ld] | value fp32 [rows]
  int ld;                  // output row length (elements)
  int n_total;             // valid outputs
  int kblocks;             // K / 64
  const int32_t* d_count;
  int count;
  int32_t* error;
};

constexpr int kDenseStages = 2;
constexpr int kDenseThreads = 192;  // TMA warp, MMA warp, 4 epilogue warps
// The fused softmax epilogue splits each 128-row tile over 16 epilogue warps (4 per TMEM lane
// quarter, 64 columns each): its per-row exponentials would otherwise run on 128 threads per
// tile, which at small batches (2 tiles for a 256-position call) sets the head's latency.
constexpr int kSoftmaxSlices = 4;
template <int MODE>
constexpr int dense_threads() { return MODE == kDenseSoftmax ? 64 + 32 * 4 * kSoftmaxSlices : kDenseThreads; }
// Shared memory requested by every dense launch: two stages of the widest tile, so that at most
// two CTAs (2 x 256 TMEM columns) share an SM.
constexpr int kDenseSmem = kDenseStages * (128 * 128 + 256 * 128) + 1024 + 256;

template <int NT, int MODE, bool F16>
__global__ void __launch_bounds__(dense_threads<MODE>())
    k_dense(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, DenseArgs a) {
  constexpr int kA = 128 * 128, kW = NT * 128;            // bytes per 64-wide K block
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;                                    // kDenseStages x (kA + kW)
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kDenseStages * (kA + kW));
  uint64_t* empty = full + kDenseStages;
  uint64_t* tfull = empty + kDenseStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int n = a.d_count ? min(*a.d_count, a.count) : a.count;
  const int row0 = blockIdx.x * 128, col0 = blockIdx.y * NT;
  if (row0 >= n) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDenseStages; ++s) { ptx::mbar_init(&full[s], 1); ptx::mbar_init(&empty[s], 1); }
    ptx::mbar_init(tfull, 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmW);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 256);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    int issued[kDenseStages] = {-1, -1};
    for (int kb = 0; kb < a.kblocks; ++kb) {
      const int s = kb % kDenseStages;
      const uint32_t ph = (uint32_t)((kb / kDenseStages) & 1);
      if (!ptx::mbar_wait(&empty[s], ph ^ 1, abort_flag, kWaitLimitNs)) break;
      ptx::mbar_arrive_expect_tx(&full[s], kA + kW);
      ptx::tma_load_2d(ring + s * (kA + kW), &tmA, &full[s], kb * kBlockK, row0);
      ptx::tma_load_2d(ring + s * (kA + kW) + kA, &tmW, &full[s], kb * kBlockK, col0);
      issued[s] = (int)ph;
    }
    for (int s = 0; s < kDenseStages; ++s)
      if (issued[s] >= 0) {
        volatile int dummy = 0;
        ptx::mbar_wait(&full[s], (uint32_t)issued[s], &dummy, kWaitLimitNs);
      }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = ptx::idesc_f16_f32(128, NT, F16);
    const uint64_t d0 = ptx::smem_desc_sw128(ptx::smem_u32(ring));
    bool ok = true;
    for (int kb = 0; kb < a.kblocks && ok; ++kb) {
      const int s = kb % kDenseStages;
      if (!ptx::mbar_wait(&full[s], (uint32_t)((kb / kDenseStages) & 1), abort_flag, kWaitLimitNs)) { ok = false; break; }
      ptx::tc_fence_after();
      const uint64_t ad = d0 + (uint64_t)(s * ((kA + kW) >> 4));
      const uint64_t wd = ad + (uint64_t)(kA >> 4);
#pragma unroll
      for (int k = 0; k < kBlockK / 16; ++k) ptx::mma_f16(tmem, ad + 2 * k, wd + 2 * k, idesc, (kb | k) != 0);
      ptx::mma_commit(&empty[s]);
    }
    ptx::mma_commit(tfull);
    // the MMAs must be complete before TMEM is freed at the end
    volatile int dummy = 0;
    ptx::mbar_wait(tfull, 0, &dummy, kWaitLimitNs);
  } else if (warp >= 2) {
    // epilogue: warp 2 + q reads TMEM lanes 32q.. (rows); one row per thread
    const int q = warp & 3;
    const int r = row0 + q * 32 + lane;
    const bool live = r < n;
    const bool ok = ptx::mbar_wait(tfull, 0, abort_flag, kWaitLimitNs);
    ptx::tc_fence_after();
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    const int ncols = min(NT, a.n_total - col0);
    if (ok && MODE == kDenseRelu16) {
      h16* out = static_cast<h16*>(a.out) + (size_t)r * a.ld + col0;
      for (int c0 = 0; c0 < NT; c0 += 32) {
        uint32_t v[32];
        ptx::tmem_ld_32x32b_x32(taddr + c0, v);
        ptx::tmem_ld_wait();
        if (live && c0 < ncols) {
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float x0 = fmaxf(__uint_as_float(v[j]) + a.bias[col0 + c0 + j], 0.f);
            const float x1 = fmaxf(__uint_as_float(v[j + 1]) + a.bias[col0 + c0 + j + 1], 0.f);
            pk[j / 2] = pack2_h16<F16>(x0, x1);
          }
          uint4* o = reinterpret_cast<uint4*>(out + c0);
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        }
      }
    } else if (ok && MODE == kDenseLogits) {
      float* out = static_cast<float*>(a.out) + (size_t)r * a.ld + col0;
      for (int c0 = 0; c0 < NT; c0 += 32) {
        uint32_t v[32];
        ptx::tmem_ld_32x32b_x32(taddr + c0, v);
        ptx::tmem_ld_wait();
        if (live) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < ncols) out[c0 + j] = __uint_as_float(v[j]) + a.bias[col0 + c0 + j];
        }
      }
    } else if (MODE == kDenseSoftmax) {
      // the whole policy row is this tile's (n_total <= NT); warp 2 + q + 4 s takes columns
      // [s * NT / 4, +NT / 4) of rows 32 q + lane: row max and exponential sums are combined over
      // the 4 slices in slice order through shared memory. Every epilogue warp reaches both
      // barriers, also after a timed-out wait (it then stores nothing).
      constexpr int kCols = NT / kSoftmaxSlices;
      static_assert(MODE != kDenseSoftmax || kDenseStages * (kA + kW) >= 4 * kSoftmaxSlices * 32 * 33 * 4,
                    "transpose buffers fit the ring");
      __shared__ float s_red[2][kSoftmaxSlices][4][32];
      const int slice = (warp - 2) >> 2;
      const int cb = slice * kCols;
      float x[kCols];
#pragma unroll
      for (int c0 = 0; c0 < kCols; c0 += 32) {
        uint32_t v[32];
        ptx::tmem_ld_32x32b_x32(taddr + cb + c0, v);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int c = cb + c0 + j;
          x[c0 + j] = (ok && c < ncols) ? __uint_as_float(v[j]) + a.bias[c] : -INFINITY;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kCols; ++j) mx = fmaxf(mx, x[j]);
      s_red[0][slice][q][lane] = mx;
      ptx::named_barrier(1, 32 * 4 * kSoftmaxSlices);
#pragma unroll
      for (int t = 0; t < kSoftmaxSlices; ++t) mx = fmaxf(mx, s_red[0][t][q][lane]);
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < kCols; ++j) {
        x[j] = (ok && cb + j < ncols) ? expf(x[j] - mx) : 0.f;
        part += x[j];
      }
      s_red[1][slice][q][lane] = part;
      ptx::named_barrier(1, 32 * 4 * kSoftmaxSlices);
      float sum = 0.f;
#pragma unroll
      for (int t = 0; t < kSoftmaxSlices; ++t) sum += s_red[1][t][q][lane];
      const float inv = 1.0f / sum;
      // stores through a 32 x 33 transpose buffer per warp (in the operand ring, idle once the
      // MMAs completed): lane l writes column l of each of the warp's 32 rows, so a warp store
      // covers 128 contiguous bytes of one row instead of one word in each of 32 rows
      float* tb = reinterpret_cast<float*>(ring) + (warp - 2) * (32 * 33);
      const int nrows = min(32, n - (row0 + q * 32));
      float* out0 = static_cast<float*>(a.out) + (size_t)(row0 + q * 32) * a.ld;
#pragma unroll
      for (int c0 = 0; c0 < kCols; c0 += 32) {
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; ++j) tb[lane * 33 + j] = x[c0 + j] * inv;
        __syncwarp();
        const int c = cb + c0 + lane;
        if (ok && c < ncols)
          for (int rr = 0; rr < nrows; ++rr) out0[(size_t)rr * a.ld + c] = tb[rr * 33 + lane];
      }
    } else if (ok && MODE == kDenseValue) {
      float acc = 0.f;
      for (int c0 = 0; c0 < NT; c0 += 32) {
        uint32_t v[32];
        ptx::tmem_ld_32x32b_x32(taddr + c0, v);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < ncols) acc += fmaxf(__uint_as_float(v[j]) + a.bias[c0 + j], 0.f) * a.w2[c0 + j];
      }
      if (live) static_cast<float*>(a.out)[r] = tanhf(acc + a.b2[0]);
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 256);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(a.error, OMQ_TIMEOUT);
}

// Softmax of fp32 logit rows in place (policies wider than one dense tile). One warp per row.
__global__ void k_softmax_rows(float* x, int ld, int n_total, const int32_t* d_count, int count) {
  const int n = d_count ? min(*d_count, count) : count;
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += gridDim.x * (blockDim.x >> 5)) {
    float* row = x + (size_t)r * ld;
    float mx = -INFINITY;
    for (int j = lane; j < n_total; j += 32) mx = fmaxf(mx, row[j]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < n_total; j += 32) sum += expf(row[j] - mx);
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    const float inv = 1.0f / sum;
    for (int j = lane; j < n_total; j += 32) row[j] = expf(row[j] - mx) * inv;
  }
}

// 1x1 convolutions (policy 2 channels, value 1) + folded BN + ReLU into the dense layers' 16-bit
// input rows: pin[pos][ch * HW + cell] (K padded, pad columns stay zero), vin[pos][cell].
__global__ void k_head_in(const h16* act, int C, int S, int P, const float* w1x1,
                          const float* b1x1, const int32_t* d_count, int count, bool f16,
                          h16* pin, int ld_p, h16* vin, int ld_v) {
  extern __shared__ float w1[];  // [3][C]
  for (int i = threadIdx.x; i < 3 * C; i += blockDim.x) w1[i] = w1x1[i];
  __syncthreads();
  const int n = d_count ? min(*d_count, count) : count;
  const int HW = S * S;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * HW; i += gridDim.x * blockDim.x) {
    const int pos = i / HW, cell = i - pos * HW;
    const int yy = cell / S, xx = cell - yy * S;
    const h16* row = act + ((size_t)pos * P + yy * (S + 1) + xx) * C;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
    for (int c = 0; c < C; c += 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + c);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
      float x[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = f16 ? unpack2_h16<true>(uw[e]) : unpack2_h16<false>(uw[e]);
        x[2 * e] = f.x;
        x[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float4 p = reinterpret_cast<const float4*>(w1 + c)[e];
        const float4 q = reinterpret_cast<const float4*>(w1 + C + c)[e];
        const float4 r = reinterpret_cast<const float4*>(w1 + 2 * C + c)[e];
        s0 += x[4 * e] * p.x + x[4 * e + 1] * p.y + x[4 * e + 2] * p.z + x[4 * e + 3] * p.w;
        s1 += x[4 * e] * q.x + x[4 * e + 1] * q.y + x[4 * e + 2] * q.z + x[4 * e + 3] * q.w;
        s2 += x[4 * e] * r.x + x[4 * e + 1] * r.y + x[4 * e + 2] * r.z + x[4 * e + 3] * r.w;
      }
    }
    pin[(size_t)pos * ld_p + cell] = to_h16(fmaxf(s0 + b1x1[0], 0.f), f16);
    pin[(size_t)pos * ld_p + HW + cell] = to_h16(fmaxf(s1 + b1x1[1], 0.f), f16);
    vin[(size_t)pos * ld_v + cell] = to_h16(fmaxf(s2 + b1x1[2], 0.f), f16);
  }
}

// Dense-layer weights W[j][k] (16-bit, K-major, zero padded to kpad columns and npad rows) from
// the fp32 head blob's transposed layout src[k][j] (k < kin, j < nout).
__global__ void k_pack_dense_w(const float* src, int kin, int nout, int kpad, int npad, bool f16, h16* dst) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < npad * kpad; i += gridDim.x * blockDim.x) {
    const int j = i / kpad, k = i - j * kpad;
    dst[i] = to_h16((j < nout && k < kin) ? src[(size_t)k * nout + j] : 0.f, f16);
  }
}

// ---------------------------------------------------------------------------------------------
// heads
// ---------------------------------------------------------------------------------------------
constexpr int kHeadPos = 8;       // positions per block
constexpr int kHeadThreads = 256;

struct HeadArgs {
  const h16* act;   // [rows][C]
  int C, S, P, A, Hp, Hv;
  const float* w1x1;          // [3][C]
  const float* b1x1;          // [3]
  const float* fc1p;          // [2*HW][Hp]
  const float* b1p;           // [Hp]
  const float* fc2p;          // [Hp][A]
  const float* b2p;           // [A]
  const float* fc1v;          // [HW][Hv]
  const float* b1v;           // [Hv]
  const float* fc2v;          // [Hv]
  const float* b2v;           // [1]
  const int32_t* d_count;
  int count;
  float* policy;              // [n][A]
  float* value;               // [n]
  bool f16;                   // activations are fp16 (else bf16)
};

// acc[p] += w * x[p] for p < HP, x 16-byte aligned in shared memory (HP / 4 broadcast loads).
template <int HP>
__device__ __forceinline__ void fma_row(float (&acc)[HP], float w, const float* x) {
#pragma unroll
  for (int i = 0; i < HP / 4; ++i) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    acc[4 * i] += w * v.x; acc[4 * i + 1] += w * v.y; acc[4 * i + 2] += w * v.z; acc[4 * i + 3] += w * v.w;
  }
}

template <int HP>
__global__ void __launch_bounds__(kHeadThreads) k_heads(HeadArgs a) {
  static_assert(HP % 4 == 0, "positions per block: a multiple of 4 (16-byte broadcast loads)");
  extern __shared__ float hsm[];
  const int HW = a.S * a.S;
  // Activations are kept position-minor ([k][8]) so that one k's 8 positions are two 16-byte
  // broadcast loads per 8 FMAs in the fully connected layers.
  float* h3 = hsm;                                // [3*HW][HP]
  float* hp = h3 + HP * 3 * HW;             // [Hp][HP]
  float* lg = hp + HP * a.Hp;               // [HP][A]
  float* hv = lg + HP * a.A;                // [HP][Hv]
  float* w1 = hv + HP * a.Hv;               // [3][C]
  const int n = a.d_count ? min(*a.d_count, a.count) : a.count;
  const int p0 = blockIdx.x * HP;
  if (p0 >= n) return;
  const int np = min(HP, n - p0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 3 * a.C; i += kHeadThreads) w1[i] = a.w1x1[i];
  // positions past the batch end compute on zeros (their outputs are not written)
  for (int i = tid; i < 3 * HW * HP; i += kHeadThreads) h3[i] = 0.f;
  __syncthreads();
  // 1x1 convolutions + folded BN + ReLU -> h3[ch*HW + cell][pos]
  for (int i = tid; i < np * HW; i += kHeadThreads) {
    const int pl = i / HW, cell = i - pl * HW;
    const int yy = cell / a.S, xx = cell - yy * a.S;
    const h16* row = a.act + ((size_t)(p0 + pl) * a.P + yy * (a.S + 1) + xx) * a.C;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
    for (int c = 0; c < a.C; c += 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + c);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
      float x[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = a.f16 ? unpack2_h16<true>(uw[e]) : unpack2_h16<false>(uw[e]);
        x[2 * e] = f.x;
        x[2 * e + 1] = f.y;
      }
      const float4* w4 = reinterpret_cast<const float4*>(w1 + c);
      const float4* w4b = reinterpret_cast<const float4*>(w1 + a.C + c);
      const float4* w4c = reinterpret_cast<const float4*>(w1 + 2 * a.C + c);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float4 p = w4[e], q = w4b[e], r = w4c[e];
        s0 += x[4 * e] * p.x + x[4 * e + 1] * p.y + x[4 * e + 2] * p.z + x[4 * e + 3] * p.w;
        s1 += x[4 * e] * q.x + x[4 * e + 1] * q.y + x[4 * e + 2] * q.z + x[4 * e + 3] * q.w;
        s2 += x[4 * e] * r.x + x[4 * e + 1] * r.y + x[4 * e + 2] * r.z + x[4 * e + 3] * r.w;
      }
    }
    h3[(size_t)cell * HP + pl] = fmaxf(s0 + a.b1x1[0], 0.f);
    h3[(size_t)(HW + cell) * HP + pl] = fmaxf(s1 + a.b1x1[1], 0.f);
    h3[(size_t)(2 * HW + cell) * HP + pl] = fmaxf(s2 + a.b1x1[2], 0.f);
  }
  __syncthreads();
  // policy fc1 (2*HW -> Hp) + ReLU
  for (int j = tid; j < a.Hp; j += kHeadThreads) {
    float acc[HP];
#pragma unroll
    for (int p = 0; p < HP; ++p) acc[p] = 0.f;
    for (int k = 0; k < 2 * HW; ++k) {
      const float w = __ldg(a.fc1p + (size_t)k * a.Hp + j);
      fma_row<HP>(acc, w, h3 + (size_t)k * HP);
    }
    const float b = a.b1p[j];
#pragma unroll
    for (int p = 0; p < HP; ++p) hp[(size_t)j * HP + p] = fmaxf(acc[p] + b, 0.f);
  }
  // value fc1 (HW -> Hv) + ReLU
  for (int j = tid; j < a.Hv; j += kHeadThreads) {
    float acc[HP];
#pragma unroll
    for (int p = 0; p < HP; ++p) acc[p] = 0.f;
    for (int k = 0; k < HW; ++k) {
      const float w = __ldg(a.fc1v + (size_t)k * a.Hv + j);
      fma_row<HP>(acc, w, h3 + (size_t)(2 * HW + k) * HP);
    }
    for (int p = 0; p < HP; ++p) hv[p * a.Hv + j] = fmaxf(acc[p] + a.b1v[j], 0.f);
  }
  __syncthreads();
  // policy fc2 (Hp -> A)
  for (int j = tid; j < a.A; j += kHeadThreads) {
    float acc[HP];
#pragma unroll
    for (int p = 0; p < HP; ++p) acc[p] = 0.f;
    for (int k = 0; k < a.Hp; ++k) {
      const float w = __ldg(a.fc2p + (size_t)k * a.A + j);
      fma_row<HP>(acc, w, hp + (size_t)k * HP);
    }
    for (int p = 0; p < HP; ++p) lg[p * a.A + j] = acc[p] + a.b2p[j];
  }
  __syncthreads();
  // softmax (= exp(log_softmax)) and value fc2 + tanh: one warp per position
  for (int p = warp; p < np; p += kHeadThreads / 32) {
    const float* l = lg + p * a.A;
    float mx = -INFINITY;
    for (int j = lane; j < a.A; j += 32) mx = fmaxf(mx, l[j]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < a.A; j += 32) sum += expf(l[j] - mx);
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    const float inv = 1.0f / sum;
    float* out = a.policy + (size_t)(p0 + p) * a.A;
    for (int j = lane; j < a.A; j += 32) out[j] = expf(l[j] - mx) * inv;
    float v = 0.f;
    for (int k = lane; k < a.Hv; k += 32) v += hv[p * a.Hv + k] * a.fc2v[k];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if (lane == 0) a.value[p0 + p] = tanhf(v + a.b2v[0]);
  }
}

}  // namespace omq

// =============================================================================================
// network object + C ABI
// =============================================================================================
using namespace omq;

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                      const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                      const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion,
                                      CUtensorMapFloatOOBfill);

struct omq_resnet {
  omq_resnet_config cfg;
  int S, P, HW, A, C, NB, Hp, Hv, max_batch;
  size_t rows;
  int sm_count;
  void* arena;
  size_t bytes;
  h16* conv_w;   // (1 + 2*NB) convs
  float* conv_b;
  float* head;
  h16* x_in;     // [rows][in_pad]
  int in_pad;              // input channels padded to 64 or 128
  h16* act[3];   // [rows][C]
  int32_t* error;
  CUtensorMap tmA_in, tmA[3], tmB_in;
  CUtensorMap tmO[3];      // output maps of the activation buffers (TMA-store epilogue)
  CUtensorMap* tmB;        // [2*NB]
  int loaded;
  // tensor-core heads (dense layers): 16-bit inputs / hidden rows / weights, their maps
  int tc_heads;
  int k1p, k3p, n1pad, n2pad, n3pad, nt3;  // padded K of fc1 policy / fc1 value, padded rows
  h16 *pin, *vin, *hid, *w1b, *w2b, *w3b;
  CUtensorMap tm_pin, tm_vin, tm_hid, tm_w1, tm_w1h, tm_w2, tm_w3;  // tm_w1h: 128-row boxes
  // whole-trunk kernel (15x15 boards, 128 filters): per-CTA scratch [3][tslots][256][128] and its
  // maps, and all residual blocks' weights as one [2 NB x 128][9 x 128] matrix
  int fused;
  int tslots;
  h16* tscratch;
  CUtensorMap tmS, tmSo, tmWall;
  bool f16;                // 16-bit storage is fp16 (OMQ_DTYPE_F16), else bf16
  // optional timing of the conv trunk of each forward call (CUDA events on the caller's stream)
  int prof_cap, prof_n;
  cudaEvent_t* prof_ev;    // [2 * prof_cap]
  int32_t* prof_counts;    // device [prof_cap]: positions evaluated by each call
  int32_t* prof_host_counts;
};

// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes) once per device (bit dev of
// `done`, so ordinals 0..63); safe when several host threads drive engines on different devices.
// An ordinal of 64 or more sets the attribute on every call.
template <class K>
static cudaError_t set_smem_attr_once(std::atomic<uint64_t>& done, K kernel, cudaFuncAttribute attr,
                                      int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, attr, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

static PFN_encodeTiled_t get_encode() {
  static PFN_encodeTiled_t fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(p);
  }
  return fn;
}

static CUtensorMapDataType map_type(bool f16) {
  return f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// 2D 16-bit tensor map for the epilogue's TMA stores: box {32 channels, 32 rows}, 64B swizzle.
static int make_out_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, bool f16) {
  PFN_encodeTiled_t enc = get_encode();
  if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return OMQ_CUDA_ERROR; }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, map_type(f16), 2, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled (output) failed (%d)", (int)r); return OMQ_CUDA_ERROR; }
  return OMQ_OK;
}

// 2D 16-bit tensor map: inner dim `inner` elements, `outer` rows, box {64, box_rows}, 128B swizzle.
static int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint32_t box_rows,
                    bool f16) {
  PFN_encodeTiled_t enc = get_encode();
  if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return OMQ_CUDA_ERROR; }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, map_type(f16), 2, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return OMQ_CUDA_ERROR; }
  return OMQ_OK;
}

// Tensor maps of a net's activation buffers and weights: activation boxes are 152-row halves of a
// tile's halo window, weight boxes 128 output channels (one work item's half of 256 filters, or all
// of 128).
static int build_maps(omq_resnet* n) {
  const uint32_t a_rows = HaloTCfg::kHaloBox;
  const uint32_t b_rows = 128;
  int st = make_map(&n->tmA_in, n->x_in, n->in_pad, n->rows, a_rows, n->f16);
  for (int i = 0; st == OMQ_OK && i < 3; ++i) st = make_map(&n->tmA[i], n->act[i], n->C, n->rows, a_rows, n->f16);
  for (int i = 0; st == OMQ_OK && i < 3; ++i) st = make_out_map(&n->tmO[i], n->act[i], n->C, n->rows, n->f16);
  if (st == OMQ_OK) st = make_map(&n->tmB_in, n->conv_w, 9 * n->in_pad, n->C, b_rows, n->f16);
  const h16* wb = n->conv_w + (size_t)n->C * 9 * n->in_pad;
  for (int i = 0; st == OMQ_OK && i < 2 * n->NB; ++i)
    st = make_map(&n->tmB[i], wb + (size_t)i * n->C * 9 * n->C, 9 * n->C, n->C, b_rows, n->f16);
  if (st == OMQ_OK && n->fused && n->tscratch) {
    const uint64_t srows = (uint64_t)3 * n->tslots * n->P;
    st = make_map(&n->tmS, n->tscratch, n->C, srows, a_rows, n->f16);
    if (st == OMQ_OK) st = make_out_map(&n->tmSo, n->tscratch, n->C, srows, n->f16);
    if (st == OMQ_OK) st = make_map(&n->tmWall, wb, 9 * n->C, (uint64_t)2 * n->NB * n->C, b_rows, n->f16);
  }
  if (st == OMQ_OK && n->tc_heads) {
    st = make_map(&n->tm_pin, n->pin, n->k1p, n->max_batch, 128, n->f16);
    if (st == OMQ_OK) st = make_map(&n->tm_vin, n->vin, n->k3p, n->max_batch, 128, n->f16);
    if (st == OMQ_OK) st = make_map(&n->tm_hid, n->hid, n->Hp, n->max_batch, 128, n->f16);
    if (st == OMQ_OK) st = make_map(&n->tm_w1, n->w1b, n->k1p, n->n1pad, 256, n->f16);
    if (st == OMQ_OK) st = make_map(&n->tm_w1h, n->w1b, n->k1p, n->n1pad, 128, n->f16);
    if (st == OMQ_OK) st = make_map(&n->tm_w2, n->w2b, n->Hp, n->n2pad, 256, n->f16);
    if (st == OMQ_OK) st = make_map(&n->tm_w3, n->w3b, n->k3p, n->n3pad, n->nt3, n->f16);
  }
  return st;
}

static size_t head_floats(const omq_resnet* n) {
  return (size_t)3 * n->C + 3 + (size_t)2 * n->HW * n->Hp + n->Hp + (size_t)n->Hp * n->A + n->A +
         (size_t)n->HW * n->Hv + n->Hv + n->Hv + 1;
}

static size_t head_smem_for(const omq_resnet* n, int hp) {
  return sizeof(float) * ((size_t)hp * (3 * n->HW + n->Hp + n->A + n->Hv) + 3 * n->C);
}
static size_t head_smem(const omq_resnet* n) { return head_smem_for(n, kHeadPos); }
// Self-test of the bounded wait every pipelined kernel here uses: one thread waits on an mbarrier
// that nothing arrives on. After limit_ns the wait gives up and raises the abort flag, and the
// kernel stores OMQ_TIMEOUT in *status and returns, leaving the context usable.
__global__ void k_selftest_wait(uint64_t limit_ns, int32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    abort_flag = 0;
    ptx::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = ptx::mbar_wait(&bar, 0, &abort_flag, limit_ns);
    *status = ok ? OMQ_OK : (abort_flag ? OMQ_TIMEOUT : OMQ_CUDA_ERROR);
  }
}

extern "C" {

int omq_resnet_create(const omq_resnet_config* cfg, omq_resnet** out) {
  if (!cfg || !out) { set_error("null argument"); return OMQ_BAD_ARG; }
  *out = nullptr;
  const omq_resnet_config c = *cfg;
  if (c.board_size < 5 || c.board_size > 19 || c.input_channels < 1 || c.input_channels > kMaxInputPlanes ||
      (c.filters != 128 && c.filters != 256) || c.num_blocks < 0 || c.num_blocks > 64 ||
      c.num_actions < 1 || c.num_actions > kMaxActions || c.fc_policy_hidden < 1 ||
      c.fc_policy_hidden > 1024 || c.fc_value_hidden < 1 || c.fc_value_hidden > 1024 ||
      c.max_batch < 1 || (c.dtype != OMQ_DTYPE_BF16 && c.dtype != OMQ_DTYPE_F16) ||
      (c.trunk_per_layer != 0 && c.trunk_per_layer != 1)) {
    set_error("bad resnet config");
    return OMQ_BAD_ARG;
  }
  DeviceGuard g(c.device);
  omq_resnet* n = new (std::nothrow) omq_resnet();
  if (!n) return OMQ_BAD_ARG;
  n->cfg = c;
  n->S = c.board_size;
  n->P = (c.board_size + 1) * (c.board_size + 1);
  n->HW = c.board_size * c.board_size;
  n->A = c.num_actions;
  n->C = c.filters;
  n->NB = c.num_blocks;
  n->Hp = c.fc_policy_hidden;
  n->Hv = c.fc_value_hidden;
  n->max_batch = c.max_batch;
  n->rows = (size_t)c.max_batch * n->P;
  n->in_pad = in_pad_of(c.input_channels);
  n->f16 = c.dtype == OMQ_DTYPE_F16;
  if (head_smem(n) > 227 * 1024) {
    set_error("heads need %zu bytes of shared memory (policy size %d)", head_smem(n), n->A);
    delete n;
    return OMQ_BAD_ARG;
  }
  cudaDeviceGetAttribute(&n->sm_count, cudaDevAttrMultiProcessorCount, c.device);
  const size_t nconv_w = (size_t)n->C * 9 * n->in_pad + (size_t)2 * n->NB * n->C * 9 * n->C;
  const size_t nconv_b = (size_t)(1 + 2 * n->NB) * n->C;
  size_t off[16], k = 0, tot = 0;
  auto take = [&](size_t b) { off[k++] = tot; tot += (b + 1023) & ~(size_t)1023; };
  take(nconv_w * 2);
  take(nconv_b * 4);
  take(head_floats(n) * 4);
  take(n->rows * n->in_pad * 2);
  for (int i = 0; i < 3; ++i) take(n->rows * n->C * 2);
  take(16);
  // tensor-core heads: fc1 width a multiple of 64 (it is the next layer's K), value width <= 256
  n->tc_heads = (n->Hp % 64 == 0 && n->Hp <= 1024 && n->Hv % 16 == 0 && n->Hv <= 256) ? 1 : 0;
  n->k1p = (2 * n->HW + 63) / 64 * 64;
  n->k3p = (n->HW + 63) / 64 * 64;
  n->n1pad = (n->Hp + 255) / 256 * 256;
  n->n2pad = (n->A + 255) / 256 * 256;
  n->nt3 = n->Hv <= 128 ? 128 : 256;
  n->n3pad = n->nt3;
  const size_t mb = (size_t)n->max_batch;
  take(n->tc_heads ? mb * n->k1p * 2 : 16);                      // 8 pin
  take(n->tc_heads ? mb * n->k3p * 2 : 16);                      // 9 vin
  take(n->tc_heads ? mb * n->Hp * 2 : 16);                       // 10 hid
  take(n->tc_heads ? (size_t)n->n1pad * n->k1p * 2 : 16);        // 11 W1
  take(n->tc_heads ? (size_t)n->n2pad * n->Hp * 2 : 16);         // 12 W2
  take(n->tc_heads ? (size_t)n->n3pad * n->k3p * 2 : 16);        // 13 W3
  n->fused = (n->P == HaloTCfg::kRows && n->C == 128 && n->NB >= 1 && n->sm_count > 0 && !c.trunk_per_layer) ? 1 : 0;
  n->tslots = n->fused ? 2 * n->sm_count : 0;
  take(n->fused ? (size_t)3 * n->tslots * n->P * n->C * 2 : 16);  // 14 trunk scratch
  void* arena = nullptr;
  cudaError_t e = cudaMalloc(&arena, tot);
  if (e != cudaSuccess) { delete n; return cuda_status(e, "cudaMalloc(resnet)"); }
  char* b = static_cast<char*>(arena);
  n->arena = arena;
  n->bytes = tot;
  n->conv_w = reinterpret_cast<h16*>(b + off[0]);
  n->conv_b = reinterpret_cast<float*>(b + off[1]);
  n->head = reinterpret_cast<float*>(b + off[2]);
  n->x_in = reinterpret_cast<h16*>(b + off[3]);
  for (int i = 0; i < 3; ++i) n->act[i] = reinterpret_cast<h16*>(b + off[4 + i]);
  n->error = reinterpret_cast<int32_t*>(b + off[7]);
  n->pin = reinterpret_cast<h16*>(b + off[8]);
  n->vin = reinterpret_cast<h16*>(b + off[9]);
  n->hid = reinterpret_cast<h16*>(b + off[10]);
  n->w1b = reinterpret_cast<h16*>(b + off[11]);
  n->w2b = reinterpret_cast<h16*>(b + off[12]);
  n->w3b = reinterpret_cast<h16*>(b + off[13]);
  n->tscratch = n->fused ? reinterpret_cast<h16*>(b + off[14]) : nullptr;
  cudaMemset(n->error, 0, 16);
  // activations start zeroed so that never-written padding rows read as zeros
  cudaMemset(b + off[3], 0, tot - off[3]);
  n->tmB = new (std::nothrow) CUtensorMap[2 * n->NB + 1];
  int st = build_maps(n);
  if (st != OMQ_OK) {
    cudaFree(arena);
    delete[] n->tmB;
    delete n;
    return st;
  }
  *out = n;
  return OMQ_OK;
}

static void prof_free(omq_resnet* n) {
  for (int i = 0; i < 2 * n->prof_cap; ++i) cudaEventDestroy(n->prof_ev[i]);
  delete[] n->prof_ev;
  delete[] n->prof_host_counts;
  if (n->prof_counts) cudaFree(n->prof_counts);
  n->prof_ev = nullptr;
  n->prof_host_counts = nullptr;
  n->prof_counts = nullptr;
  n->prof_cap = n->prof_n = 0;
}

int omq_resnet_destroy(omq_resnet* n) {
  if (!n) return OMQ_OK;
  DeviceGuard g(n->cfg.device);
  prof_free(n);
  cudaError_t e = cudaFree(n->arena);
  delete[] n->tmB;
  delete n;
  return cuda_status(e, "cudaFree(resnet)");
}

int omq_resnet_param_sizes(const omq_resnet* n, uint64_t* conv_w, uint64_t* conv_b, uint64_t* head) {
  if (!n) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (conv_w) *conv_w = (uint64_t)n->C * 9 * n->in_pad + (uint64_t)2 * n->NB * n->C * 9 * n->C;
  if (conv_b) *conv_b = (uint64_t)(1 + 2 * n->NB) * n->C;
  if (head) *head = head_floats(n);
  return OMQ_OK;
}

int omq_resnet_load(omq_resnet* n, const uint16_t* d_conv_w, const float* d_conv_b,
                    const float* d_head, void* stream) {
  if (!n || !d_conv_w || !d_conv_b || !d_head) { set_error("null argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(n->cfg.device);
  uint64_t a, b, h;
  omq_resnet_param_sizes(n, &a, &b, &h);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(n->conv_w, d_conv_w, a * 2, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(n->conv_b, d_conv_b, b * 4, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(n->head, d_head, h * 4, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return cuda_status(e, "omq_resnet_load");
  if (n->tc_heads) {
    // the dense layers' bf16 weights [out][in], from the blob's transposed fp32 layouts
    const float* p = n->head + 3 * n->C + 3;
    const float* fc1p = p;
    const float* fc2p = fc1p + (size_t)2 * n->HW * n->Hp + n->Hp;
    const float* fc1v = fc2p + (size_t)n->Hp * n->A + n->A;
    count_launches(3);
    k_pack_dense_w<<<256, 256, 0, s>>>(fc1p, 2 * n->HW, n->Hp, n->k1p, n->n1pad, n->f16, n->w1b);
    k_pack_dense_w<<<256, 256, 0, s>>>(fc2p, n->Hp, n->A, n->Hp, n->n2pad, n->f16, n->w2b);
    k_pack_dense_w<<<256, 256, 0, s>>>(fc1v, n->HW, n->Hv, n->k3p, n->n3pad, n->f16, n->w3b);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "omq_resnet_load: dense weights");
  }
  n->loaded = 1;
  return OMQ_OK;
}

int omq_resnet_trunk_launches(const omq_resnet* n, int32_t* launches) {
  if (!n || !launches) { set_error("null argument"); return OMQ_BAD_ARG; }
  *launches = (n->fused && n->tscratch) ? 1 : 1 + 2 * n->NB;
  return OMQ_OK;
}

int omq_resnet_memory(const omq_resnet* n, uint64_t* bytes) {
  if (!n || !bytes) { set_error("null argument"); return OMQ_BAD_ARG; }
  *bytes = n->bytes;
  return OMQ_OK;
}

}  // extern "C"

namespace omq {

template <bool F16>
static int launch_conv_halo_tr(const omq_resnet* n, const CUtensorMap& tH, const CUtensorMap& tB,
                               const CUtensorMap& tO, const ConvArgs& a, cudaStream_t s) {
  static std::atomic<uint64_t> attr_set{0};
  {
    const cudaError_t e = set_smem_attr_once(attr_set, k_conv3x3_halo_t<F16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, HaloTCfg::kSmem);
    if (e != cudaSuccess) return cuda_status(e, "transposed halo conv smem attribute");
  }
  const int max_items = (int)((n->rows + HaloTCfg::kRows - 1) / HaloTCfg::kRows) * a.halves;
  const int grid = max(1, min(max_items, n->sm_count));
  count_launches(1);
  // programmatic dependent launch: the CTAs may start (and run their setup) while the previous
  // kernel's last CTAs finish; the kernel waits for that kernel before touching global memory
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(HaloTCfg::kThreads);
  cfg.dynamicSmemBytes = HaloTCfg::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, k_conv3x3_halo_t<F16>, tH, tB, tO, a), "k_conv3x3_halo_t");
}

template <bool F16>
static int launch_trunk_t(const omq_resnet* n, const TrunkArgs& a, cudaStream_t s) {
  static std::atomic<uint64_t> attr_set{0};
  {
    const cudaError_t e = set_smem_attr_once(attr_set, k_trunk_t<F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             HaloTCfg::kSmem);
    if (e != cudaSuccess) return cuda_status(e, "trunk kernel smem attribute");
  }
  count_launches(1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n->sm_count);
  cfg.blockDim = dim3(HaloTCfg::kThreads);
  cfg.dynamicSmemBytes = HaloTCfg::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, k_trunk_t<F16>, n->tmA_in, n->tmB_in, n->tmWall, n->tmS, n->tmSo,
                                        n->tmO[0], a),
                     "k_trunk_t");
}

// The whole trunk in one launch (k_trunk_t); the output lands in act[0].
static int trunk(const omq_resnet* n, const int32_t* d_count, int count, cudaStream_t s) {
  TrunkArgs a{n->conv_b, n->tscratch, d_count, count, 1 + 2 * n->NB, n->in_pad / kBlockK, 2 * n->sm_count,
              n->error};
  return n->f16 ? launch_trunk_t<true>(n, a, s) : launch_trunk_t<false>(n, a, s);
}

static int conv(const omq_resnet* n, const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tO,
                const float* bias,
                const h16* res, h16* out, int kb_per_tap, const int32_t* d_count,
                int count, cudaStream_t s) {
  const ConvArgs a{bias, res, out, d_count, count, n->P, n->S, kb_per_tap, 1, n->error, n->C / 128};
  return n->f16 ? launch_conv_halo_tr<true>(n, tA, tB, tO, a, s) : launch_conv_halo_tr<false>(n, tA, tB, tO, a, s);
}

template <int NT, int MODE, bool F16>
static int launch_dense_t(const CUtensorMap& tA, const CUtensorMap& tW, const DenseArgs& a, int rows_cap,
                          int ntiles, cudaStream_t s) {
  static std::atomic<uint64_t> attr_set{0};
  {
    const cudaError_t e = set_smem_attr_once(attr_set, k_dense<NT, MODE, F16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kDenseSmem);
    if (e != cudaSuccess) return cuda_status(e, "dense smem attribute");
  }
  count_launches(1);
  k_dense<NT, MODE, F16><<<dim3((rows_cap + 127) / 128, ntiles), dense_threads<MODE>(), kDenseSmem, s>>>(tA, tW, a);
  return cuda_status(cudaGetLastError(), "k_dense");
}

template <int NT, int MODE>
static int launch_dense(const omq_resnet* n, const CUtensorMap& tA, const CUtensorMap& tW, const DenseArgs& a,
                        int rows_cap, int ntiles, cudaStream_t s) {
  return n->f16 ? launch_dense_t<NT, MODE, true>(tA, tW, a, rows_cap, ntiles, s)
                : launch_dense_t<NT, MODE, false>(tA, tW, a, rows_cap, ntiles, s);
}

// Heads on the tensor cores: 1x1 convolutions -> 16-bit rows, then fc1 (policy) with ReLU,
// fc2 (policy) with the softmax fused when the policy fits one 256-wide tile, and the value
// head's fc1 with the fc2 dot and tanh fused.
static int run_tc_heads(omq_resnet* n, const h16* act, const int32_t* d_count, int count,
                        float* policy, float* value, bool value_only, cudaStream_t s) {
  const float* p = n->head;
  const float* w1x1 = p; p += 3 * n->C;
  const float* b1x1 = p; p += 3;
  p += (size_t)2 * n->HW * n->Hp;
  const float* b1p = p; p += n->Hp;
  p += (size_t)n->Hp * n->A;
  const float* b2p = p; p += n->A;
  p += (size_t)n->HW * n->Hv;
  const float* b1v = p; p += n->Hv;
  const float* fc2v = p; p += n->Hv;
  const float* b2v = p;
  count_launches(1);
  k_head_in<<<max(1, min((count * n->HW + 255) / 256, 4 * n->sm_count)), 256, 3 * n->C * sizeof(float), s>>>(
      act, n->C, n->S, n->P, w1x1, b1x1, d_count, count, n->f16, n->pin, n->k1p, n->vin, n->k3p);
  int st = cuda_status(cudaGetLastError(), "k_head_in");
  if (st) return st;
  DenseArgs a{};
  a.d_count = d_count;
  a.count = count;
  a.error = n->error;
  if (!value_only) {
    // policy fc1 -> hidden (16-bit, ReLU)
    a.bias = b1p; a.out = n->hid; a.ld = n->Hp; a.n_total = n->Hp; a.kblocks = n->k1p / 64;
    // a batch that fills fewer than half the SMs with 256-wide tiles takes 128-wide ones (twice the
    // CTAs, each loading half the weights; the K loop is the same, so are the results)
    if ((count + 127) / 128 * (n->n1pad / 256) * 2 <= n->sm_count)
      st = launch_dense<128, kDenseRelu16>(n, n->tm_pin, n->tm_w1h, a, count, n->n1pad / 128, s);
    else
      st = launch_dense<256, kDenseRelu16>(n, n->tm_pin, n->tm_w1, a, count, n->n1pad / 256, s);
    if (st) return st;
    // policy fc2 -> probabilities
    a.bias = b2p; a.out = policy; a.ld = n->A; a.n_total = n->A; a.kblocks = n->Hp / 64;
    if (n->A <= 256) {
      st = launch_dense<256, kDenseSoftmax>(n, n->tm_hid, n->tm_w2, a, count, 1, s);
    } else {
      st = launch_dense<256, kDenseLogits>(n, n->tm_hid, n->tm_w2, a, count, n->n2pad / 256, s);
      if (!st) {
        count_launches(1);
        k_softmax_rows<<<max(1, min((count + 7) / 8, 8 * n->sm_count)), 256, 0, s>>>(policy, n->A, n->A, d_count, count);
        st = cuda_status(cudaGetLastError(), "k_softmax_rows");
      }
    }
    if (st) return st;
  }
  // value fc1 + ReLU, fc2, tanh
  a.bias = b1v; a.w2 = fc2v; a.b2 = b2v; a.out = value; a.ld = 1; a.n_total = n->Hv; a.kblocks = n->k3p / 64;
  if (n->nt3 == 128) return launch_dense<128, kDenseValue>(n, n->tm_vin, n->tm_w3, a, count, 1, s);
  return launch_dense<256, kDenseValue>(n, n->tm_vin, n->tm_w3, a, count, 1, s);
}

// trunk + heads on n->x_in (already packed), count from d_count (device) or `count`.
int resnet_run(omq_resnet* n, const int32_t* d_count, int count, float* policy, float* value,
               cudaStream_t s, bool value_only = false) {
  if (!n->loaded) { set_error("omq_resnet_load was not called"); return OMQ_NOT_READY; }
  const int pi = (n->prof_cap > 0 && n->prof_n < n->prof_cap) ? n->prof_n++ : -1;
  if (pi >= 0) {
    if (d_count)
      cudaMemcpyAsync(n->prof_counts + pi, d_count, 4, cudaMemcpyDeviceToDevice, s);
    else
      n->prof_host_counts[pi] = count;
    cudaEventRecord(n->prof_ev[2 * pi], s);
  }
  int st = OMQ_OK;
  int x = 0;
  if (n->fused && n->tscratch) {
    st = trunk(n, d_count, count, s);  // output in act[0]
  } else {
    st = conv(n, n->tmA_in, n->tmB_in, n->tmO[0], n->conv_b, nullptr, n->act[0], n->in_pad / kBlockK,
              d_count, count, s);
  }
  for (int i = 0; !(n->fused && n->tscratch) && st == OMQ_OK && i < n->NB; ++i) {
    const int t = (x + 1) % 3, y = (x + 2) % 3;
    st = conv(n, n->tmA[x], n->tmB[2 * i], n->tmO[t], n->conv_b + (size_t)(1 + 2 * i) * n->C, nullptr,
              n->act[t], n->C / kBlockK, d_count, count, s);
    if (st) break;
    st = conv(n, n->tmA[t], n->tmB[2 * i + 1], n->tmO[y], n->conv_b + (size_t)(2 + 2 * i) * n->C, n->act[x],
              n->act[y], n->C / kBlockK, d_count, count, s);
    x = y;
  }
  if (st) return st;
  if (pi >= 0) cudaEventRecord(n->prof_ev[2 * pi + 1], s);
  if (n->tc_heads) return run_tc_heads(n, n->act[x], d_count, count, policy, value, value_only, s);
  HeadArgs h{};
  h.act = n->act[x];
  h.C = n->C; h.S = n->S; h.P = n->P; h.A = n->A; h.Hp = n->Hp; h.Hv = n->Hv;
  const float* p = n->head;
  h.w1x1 = p; p += 3 * n->C;
  h.b1x1 = p; p += 3;
  h.fc1p = p; p += (size_t)2 * n->HW * n->Hp;
  h.b1p = p; p += n->Hp;
  h.fc2p = p; p += (size_t)n->Hp * n->A;
  h.b2p = p; p += n->A;
  h.fc1v = p; p += (size_t)n->HW * n->Hv;
  h.b1v = p; p += n->Hv;
  h.fc2v = p; p += n->Hv;
  h.b2v = p;
  h.d_count = d_count;
  h.count = count;
  h.policy = policy;
  h.value = value;
  h.f16 = n->f16;
  const size_t sm = head_smem_for(n, kHeadPos);
  cudaError_t e = cudaFuncSetAttribute(k_heads<kHeadPos>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return cuda_status(e, "heads smem attribute");
  const int blocks = (count + kHeadPos - 1) / kHeadPos;
  count_launches(1);
  k_heads<kHeadPos><<<blocks, kHeadThreads, sm, s>>>(h);
  return cuda_status(cudaGetLastError(), "k_heads");
}

}  // namespace omq

extern "C" {

int omq_resnet_forward_features(omq_resnet* n, const float* d_features, int32_t batch,
                                float* d_policy, float* d_value, void* stream) {
  if (!n || !d_features || !d_policy || !d_value) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (batch < 0 || batch > n->max_batch) {
    set_error("batch %d outside [0, %d]", batch, n->max_batch);
    return OMQ_BAD_ARG;
  }
  if (batch == 0) return OMQ_OK;
  DeviceGuard g(n->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  const int total = batch * n->P * (n->in_pad / 8);
  count_launches(1);
  k_pack_features<<<min((total + 255) / 256, 8192), 256, 0, s>>>(
      d_features, n->cfg.input_channels, n->S, n->P, nullptr, batch, n->f16, n->x_in);
  int st = cuda_status(cudaGetLastError(), "k_pack_features");
  if (st) return st;
  return resnet_run(n, nullptr, batch, d_policy, d_value, s);
}

int omq_resnet_forward_packed(omq_resnet* n, const uint16_t* d_input, const int32_t* d_count,
                              int32_t batch, float* d_policy, float* d_value, void* stream) {
  if (!n || !d_policy || !d_value) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (batch < 0 || batch > n->max_batch) { set_error("batch outside capacity"); return OMQ_BAD_ARG; }
  DeviceGuard g(n->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  if (d_input && d_input != reinterpret_cast<const uint16_t*>(n->x_in)) {
    cudaError_t e = cudaMemcpyAsync(n->x_in, d_input, (size_t)batch * n->P * n->in_pad * 2,
                                    cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_status(e, "omq_resnet_forward_packed copy");
  }
  return resnet_run(n, d_count, batch, d_policy, d_value, s);
}

int omq_resnet_input_buffer(omq_resnet* n, uint16_t** d_input) {
  if (!n || !d_input) { set_error("null argument"); return OMQ_BAD_ARG; }
  *d_input = reinterpret_cast<uint16_t*>(n->x_in);
  return OMQ_OK;
}

int omq_resnet_forward_queue(omq_resnet* n, omq_engine* e, int32_t queue, void* stream) {
  if (!n || !e || queue < 0 || queue > 1) { set_error("bad argument"); return OMQ_BAD_ARG; }
  const int cap = e->v.R * e->v.WCAP;
  if (n->max_batch < cap) {
    set_error("resnet max_batch %d < engine queue capacity %d", n->max_batch, cap);
    return OMQ_BAD_ARG;
  }
  if (n->S != e->v.S || n->A != e->v.A || n->cfg.input_channels != engine_planes(e->v)) {
    set_error("resnet / engine mismatch: board %d/%d, actions %d/%d, planes %d/%d", n->S, e->v.S,
              n->A, e->v.A, n->cfg.input_channels, engine_planes(e->v));
    return OMQ_BAD_ARG;
  }
  DeviceGuard g(n->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  launch_pack_queue(e->v, queue, n->P, n->in_pad, n->x_in, n->f16, s);
  int st = cuda_status(cudaGetLastError(), "pack queue");
  if (st) return st;
  // the final-node queue's policies are never read by the search (the reference discards them,
  // wave_search.py:1337-1457): its forward stops after the value head
  return resnet_run(n, e->v.q_count + queue, cap, e->v.q_policy[queue], e->v.q_value[queue], s, queue == 1);
}

int omq_resnet_profile(omq_resnet* n, int32_t capacity) {
  if (!n || capacity < 0 || capacity > (1 << 20)) { set_error("bad argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(n->cfg.device);
  prof_free(n);
  if (capacity == 0) return OMQ_OK;
  n->prof_ev = new (std::nothrow) cudaEvent_t[2 * capacity];
  n->prof_host_counts = new (std::nothrow) int32_t[capacity];
  if (!n->prof_ev || !n->prof_host_counts) { set_error("host allocation failed"); return OMQ_BAD_ARG; }
  for (int i = 0; i < 2 * capacity; ++i) cudaEventCreate(&n->prof_ev[i]);
  cudaError_t e = cudaMalloc(&n->prof_counts, 4 * (size_t)capacity);
  if (e == cudaSuccess) e = cudaMemset(n->prof_counts, 0xFF, 4 * (size_t)capacity);
  n->prof_cap = capacity;
  for (int i = 0; i < capacity; ++i) n->prof_host_counts[i] = -1;
  return cuda_status(e, "omq_resnet_profile");
}

int omq_resnet_profile_read(omq_resnet* n, int32_t* h_calls, float* h_trunk_ms, int32_t* h_counts,
                            int32_t max) {
  if (!n || !h_calls) { set_error("null argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(n->cfg.device);
  const int k = n->prof_n < max ? n->prof_n : max;
  *h_calls = k;
  if (k == 0) return OMQ_OK;
  cudaError_t e = cudaEventSynchronize(n->prof_ev[2 * (k - 1) + 1]);
  for (int i = 0; e == cudaSuccess && i < k; ++i)
    if (h_trunk_ms) e = cudaEventElapsedTime(&h_trunk_ms[i], n->prof_ev[2 * i], n->prof_ev[2 * i + 1]);
  if (e == cudaSuccess && h_counts) {
    e = cudaMemcpy(h_counts, n->prof_counts, 4 * (size_t)k, cudaMemcpyDeviceToHost);
    for (int i = 0; i < k; ++i)
      if (n->prof_host_counts[i] >= 0) h_counts[i] = n->prof_host_counts[i];
  }
  return cuda_status(e, "omq_resnet_profile_read");
}

int omq_selftest_wait_timeout(uint64_t limit_ns, int32_t* d_status, void* stream) {
  if (!d_status || limit_ns == 0 || limit_ns > 1000000000ull) {
    set_error("omq_selftest_wait_timeout: d_status null or limit outside (0, 1 s]");
    return OMQ_BAD_ARG;
  }
  count_launches(1);
  k_selftest_wait<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns, d_status);
  return cuda_status(cudaGetLastError(), "k_selftest_wait");
}

int omq_resnet_error(omq_resnet* n, int32_t* h_error, void* stream) {
  if (!n || !h_error) { set_error("null argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(n->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(h_error, n->error, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return cuda_status(e, "omq_resnet_error");
}

}  // extern "C"

// =============================================================================================
// Forward pass that allocates nothing
// =============================================================================================
// Some callers cannot let a library call cudaMalloc: processes whose own memory manager owns the
// whole device heap (a serving process that reserves all of HBM for its pool up front), and
// latency-critical threads, where cudaMalloc / cudaFree would synchronise the device and stall
// every other stream. omq_resnet_forward_noalloc serves them: the caller passes the packed
// weights, the input features and the output buffers, and the activations live in one fixed
// device array compiled into this library. That array (kNoAllocScratchBytes) is held by every
// GPU that loads the library until the process exits, and every call shares it.
namespace omq {
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB of activations + the error word
}
static __device__ __align__(256) uint8_t g_noalloc_scratch[omq::kNoAllocScratchBytes];

namespace omq {
constexpr int kMaxDevices = 64;
// Device address of g_noalloc_scratch per device ordinal, looked up once per device with that
// device current. In host code the array's name is only a host-side stand-in, never a usable
// device address. Threads that race on a first lookup store the same address.
static std::atomic<uint8_t*> g_noalloc_ptr[kMaxDevices];

// Makes `dev` current (the caller's DeviceGuard restores the previous device) and returns the
// scratch array's device address on it.
static int noalloc_scratch(int dev, uint8_t** out) {
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceCount");
  if (dev < 0 || dev >= ndev || dev >= kMaxDevices) {
    set_error("device ordinal %d out of range (%d devices)", dev, ndev);
    return OMQ_BAD_ARG;
  }
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  uint8_t* p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    void* q = nullptr;
    e = cudaGetSymbolAddress(&q, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(no-alloc scratch)");
    p = static_cast<uint8_t*>(q);
    g_noalloc_ptr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return OMQ_OK;
}
// The error word sits in the last 256 bytes of the scratch, clear of the activations.
constexpr size_t kNoAllocErrorOffset = kNoAllocScratchBytes - 256;
}  // namespace omq

extern "C" int omq_resnet_forward_noalloc(const omq_resnet_config* cfg, const uint16_t* d_conv_w,
                                          const float* d_conv_b, const float* d_head,
                                          const float* d_features, int32_t batch,
                                          float* d_policy, float* d_value, void* stream) {
  if (!cfg || !d_conv_w || !d_conv_b || !d_head || !d_features || !d_policy || !d_value) {
    set_error("null argument");
    return OMQ_BAD_ARG;
  }
  const omq_resnet_config c = *cfg;
  if (c.board_size < 5 || c.board_size > 19 || c.input_channels < 1 || c.input_channels > kMaxInputPlanes ||
      (c.filters != 128 && c.filters != 256) || c.num_blocks < 0 || c.num_blocks > 64 ||
      c.num_actions < 1 || c.num_actions > kMaxActions || c.fc_policy_hidden < 1 ||
      c.fc_policy_hidden > 1024 || c.fc_value_hidden < 1 || c.fc_value_hidden > 1024 ||
      (c.dtype != OMQ_DTYPE_BF16 && c.dtype != OMQ_DTYPE_F16)) {
    set_error("bad resnet config");
    return OMQ_BAD_ARG;
  }
  const int P = (c.board_size + 1) * (c.board_size + 1);
  // scratch: the packed input [rows][64] + three activation buffers [rows][F] (bf16) + error word
  const int in_pad = in_pad_of(c.input_channels);
  const size_t per_pos = (size_t)P * (in_pad + 3 * (size_t)c.filters) * 2;
  const int max_batch = (int)((kNoAllocScratchBytes - 1024) / per_pos);
  if (batch < 0 || batch > max_batch) {
    set_error("omq_resnet_forward_noalloc: batch %d exceeds the fixed scratch limit of %d positions "
              "(%zu-byte scratch, %d filters)", batch, max_batch, kNoAllocScratchBytes, c.filters);
    return OMQ_BAD_ARG;
  }
  if (batch == 0) return OMQ_OK;
  DeviceGuard g(c.device);
  uint8_t* base = nullptr;
  int st = noalloc_scratch(c.device, &base);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  // a view of the library's net object over caller weights and the fixed scratch (host stack only)
  omq_resnet n{};
  CUtensorMap maps[2 * 64];
  n.cfg = c;
  n.S = c.board_size;
  n.P = P;
  n.HW = c.board_size * c.board_size;
  n.A = c.num_actions;
  n.C = c.filters;
  n.NB = c.num_blocks;
  n.Hp = c.fc_policy_hidden;
  n.Hv = c.fc_value_hidden;
  n.max_batch = max_batch;
  n.rows = (size_t)max_batch * P;
  n.in_pad = in_pad;
  n.f16 = c.dtype == OMQ_DTYPE_F16;
  if (head_smem(&n) > 227 * 1024) { set_error("heads need too much shared memory"); return OMQ_BAD_ARG; }
  cudaDeviceGetAttribute(&n.sm_count, cudaDevAttrMultiProcessorCount, c.device);
  n.conv_w = reinterpret_cast<h16*>(const_cast<uint16_t*>(d_conv_w));
  n.conv_b = const_cast<float*>(d_conv_b);
  n.head = const_cast<float*>(d_head);
  n.x_in = reinterpret_cast<h16*>(base);
  size_t off = ((n.rows * in_pad * 2) + 255) & ~(size_t)255;
  for (int i = 0; i < 3; ++i) {
    n.act[i] = reinterpret_cast<h16*>(base + off);
    off += ((n.rows * n.C * 2) + 255) & ~(size_t)255;
  }
  n.error = reinterpret_cast<int32_t*>(base + kNoAllocErrorOffset);
  n.tmB = maps;
  n.loaded = 1;
  st = build_maps(&n);
  if (st) return st;
  // the error word keeps the previous call's value: clear it
  cudaError_t e = cudaMemsetAsync(n.error, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_status(e, "omq_resnet_forward_noalloc: clearing the error word");
  const int total = batch * P * (in_pad / 8);
  count_launches(1);
  k_pack_features<<<min((total + 255) / 256, 8192), 256, 0, s>>>(
      d_features, c.input_channels, n.S, P, nullptr, batch, n.f16, n.x_in);
  st = cuda_status(cudaGetLastError(), "k_pack_features");
  if (st) return st;
  return resnet_run(&n, nullptr, batch, d_policy, d_value, s);
}

// Reads the error word of the last omq_resnet_forward_noalloc call on `device` (OMQ_OK, or
// OMQ_TIMEOUT when a pipelined kernel's bounded wait gave up) after the work queued on `stream`.
// Like the forward itself, it allocates nothing: the word is copied into the caller's int.
extern "C" int omq_resnet_noalloc_error(int32_t device, int32_t* h_error, void* stream) {
  if (!h_error) { set_error("null argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(device);
  uint8_t* base = nullptr;
  int st = omq::noalloc_scratch(device, &base);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(h_error, base + omq::kNoAllocErrorOffset, sizeof(int32_t),
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return cuda_status(e, "omq_resnet_noalloc_error");
}
