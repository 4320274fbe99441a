// C ABI of libcea.so: argument checking, kernel selection, TMA descriptors, launches.
//
// Everything is stream-ordered; no entry point synchronises the host (except
// cea_device_status, which exists to do exactly that) or allocates memory.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

#include "attn_f32.cuh"
#include "attn_simt.cuh"
#include "attn_tc2.cuh"
#include "cea_common.cuh"
#include "cea_nccl.cuh"
#include "decode.cuh"
#include "kv_cache.cuh"
#include "wire.cuh"
#include "llama_ops.cuh"
#include "peer_merge.cuh"

using namespace cea;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CEA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return CEA_OK;
}

// ---------------------------------------------------------------- TMA maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [B, S, H, D] 16-bit tensor (D contiguous) as a 4-D tensor map with a (64, rows, 1, 1) box, 128B swizzle
bool make_map(CUtensorMap* map, int dtype, const void* ptr, int D, int S, int H, int B, int64_t ss, int64_t sh,
              int64_t sb, int rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  // strides of size-1 dimensions are never used: give them any legal value
  if (H == 1) sh = ss;
  if (B == 1) sb = ss;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss) * 2, static_cast<cuuint64_t>(sh) * 2,
                                 static_cast<cuuint64_t>(sb) * 2};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(rows), 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType t =
      dtype == CEA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, t, 4, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// a [B, S, H, D] 16-bit operand TMA can read: 16-byte aligned base, strides multiples of 8 elements
bool tma_ok(const void* ptr, const int64_t* st, int S, int H, int B) {
  if (!aligned16(ptr)) return false;
  const int64_t ss = st[1], sh = H == 1 ? st[1] : st[2], sb = B == 1 ? st[1] : st[0];
  for (int64_t s : {ss, sh, sb})
    if (s <= 0 || (s % 8) != 0 || s * 2 >= (int64_t(1) << 40)) return false;
  (void)S;
  return true;
}

int elem_bytes(int dt) { return dt == CEA_F64 ? 8 : (dt == CEA_F32 ? 4 : 2); }

int num_sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

int validate(const cea_attn_params* p) {
  if (p == nullptr) return fail(CEA_ERR_INVALID, "null params");
  if (p->B < 0 || p->Sq < 0 || p->Sk < 0 || p->Hq < 0 || p->Hkv < 1 || p->D < 1)
    return fail(CEA_ERR_INVALID, "invalid sizes B=%d Sq=%d Sk=%d Hq=%d Hkv=%d D=%d", p->B, p->Sq, p->Sk, p->Hq, p->Hkv,
                p->D);
  if (p->kv_map == nullptr && p->Hq % p->Hkv != 0)
    return fail(CEA_ERR_INVALID, "%d query heads cannot share %d KV heads evenly", p->Hq, p->Hkv);
  const int in = p->in_dtype, out = p->out_dtype;
  if (in < CEA_F32 || in > CEA_F64) return fail(CEA_ERR_INVALID, "unknown input dtype %d", in);
  const bool out_ok = in == CEA_F64 ? (out == CEA_F64) : (out == CEA_F32 || out == in);
  if (!out_ok) return fail(CEA_ERR_UNSUPPORTED, "output dtype %d not available for input dtype %d", out, in);
  const bool wide_out = out == CEA_F32 || out == CEA_F64;
  if (p->acc_in != nullptr && (!p->accumulate || wide_out))
    return fail(CEA_ERR_INVALID, "acc_in serves accumulate = 1 with a 16-bit output only");
  if (p->accumulate && (p->lse == nullptr || (!wide_out && p->acc_in == nullptr)))
    return fail(CEA_ERR_INVALID, "accumulate needs lse and an fp32/fp64 output (or acc_in)");
  if (p->acc_in != nullptr && p->Sk == 0)
    return fail(CEA_ERR_UNSUPPORTED, "acc_in with no keys: nothing to merge, copy acc_in to out instead");
  const bool empty = p->B == 0 || p->Sq == 0 || p->Hq == 0;
  if (!empty && (p->out == nullptr || p->q_pos == nullptr || p->q == nullptr))
    return fail(CEA_ERR_INVALID, "null q, out or q_pos");
  if (!empty && p->Sk > 0 && (p->k == nullptr || p->v == nullptr || p->k_pos == nullptr))
    return fail(CEA_ERR_INVALID, "null k, v or k_pos");
  if (p->n_new < 0 || p->n_new > p->Sk)
    return fail(CEA_ERR_INVALID, "n_new = %d new tokens do not fit the %d keys", p->n_new, p->Sk);
  if (p->n_new > 0 && (p->new_k == nullptr || p->new_v == nullptr || p->new_pos == nullptr))
    return fail(CEA_ERR_INVALID, "null new_k, new_v or new_pos with n_new = %d", p->n_new);
  return CEA_OK;
}

// the decode kernel copies the new tokens' rows in 16-byte units
bool append_ok(const cea_attn_params* p) {
  if (p->n_new == 0) return true;
  if (!aligned16(p->new_k) || !aligned16(p->new_v)) return false;
  for (int i = 0; i < 3; ++i)
    if ((p->new_k_stride[i] % 8) != 0 || (p->new_v_stride[i] % 8) != 0) return false;
  return true;
}

enum Kind { kNone = 0, kTc = 1, kDecode = 2, kSimt = 3 };

bool decode_ok(const cea_attn_params* p) {
  if (p->acc_in != nullptr) return false;
  if (p->in_dtype != CEA_BF16 && p->in_dtype != CEA_F16) return false;
  if (p->D != 64 && p->D != 128) return false;
  if (p->kv_map != nullptr) return false;
  const int G = p->Hq / p->Hkv;
  if (static_cast<int64_t>(p->Sq) * G > dec::MAX_ROWS) return false;
  if ((reinterpret_cast<uintptr_t>(p->q) & 3u) != 0 || (p->q_stride[0] | p->q_stride[1] | p->q_stride[2]) & 1) return false;
  if (!append_ok(p)) return false;
  return tma_ok(p->k, p->k_stride, p->Sk, p->Hkv, p->B) && tma_ok(p->v, p->v_stride, p->Sk, p->Hkv, p->B);
}

bool tc_ok(const cea_attn_params* p) {
  if (p->in_dtype != CEA_BF16 && p->in_dtype != CEA_F16) return false;
  if (p->D != 64 && p->D != 128) return false;
  if (!tma_ok(p->q, p->q_stride, p->Sq, p->Hq, p->B) || !tma_ok(p->k, p->k_stride, p->Sk, p->Hkv, p->B) ||
      !tma_ok(p->v, p->v_stride, p->Sk, p->Hkv, p->B))
    return false;
  // the epilogue stores 16-byte vectors of a row
  const int vec = p->out_dtype == CEA_F32 ? 4 : 8;
  if (!aligned16(p->out)) return false;
  for (int i = 0; i < 3; ++i)
    if (p->o_stride[i] % vec) return false;
  if (p->acc_in != nullptr) {  // fp32 rows read as 16-byte vectors
    if (!aligned16(p->acc_in)) return false;
    for (int i = 0; i < 3; ++i)
      if (p->acc_stride[i] % 4) return false;
  }
  return true;
}

int select_kind(const cea_attn_params* p) {
  if (p->B == 0 || p->Sq == 0 || p->Hq == 0 || p->Sk == 0) return kNone;
  if (p->acc_in != nullptr) return tc_ok(p) ? kTc : kSimt;  // only the tcgen05 epilogue reads acc_in
  if (decode_ok(p)) return kDecode;
  if (tc_ok(p)) return kTc;
  return kSimt;
}

// ---------------------------------------------------------------- decode sizing
struct DecodePlan {
  int nsplit, tiles_per_split;
  size_t part_bytes;
};

// max_bytes bounds the partials' size (the fixed scratch of cea_decode_splitkv_noalloc);
// nsplit is 0 when not even one split fits
DecodePlan decode_plan(const cea_attn_params* p, size_t max_bytes = SIZE_MAX) {
  const int nkt = (p->Sk + dec::BKEYS - 1) / dec::BKEYS;
  const int per_sm = p->D == 128 ? 2 : 3;  // resident CTAs per SM (shared-memory bound)
  const int slots = num_sms() * per_sm;
  const int64_t pairs = static_cast<int64_t>(p->B) * p->Hkv;
  const size_t split_bytes = static_cast<size_t>(p->B) * p->Hq * p->Sq * (p->D + 1) * sizeof(float);
  const size_t fit = split_bytes ? max_bytes / split_bytes : 0;
  // pick the split count minimising (waves x tiles per split), preferring fewer splits on ties
  int best = 1;
  double best_cost = 1e30;
  const int max_split = std::max(1, std::min(std::min(256, nkt), static_cast<int>(std::min<size_t>(fit, 256))));
  if (fit == 0) return DecodePlan{0, 0, split_bytes};
  for (int ns = 1; ns <= max_split; ++ns) {
    const int tps = (nkt + ns - 1) / ns;
    const int used = (nkt + tps - 1) / tps;
    if (used != ns) continue;  // this split count leaves empty splits
    const int64_t ctas = pairs * ns;
    const double waves = static_cast<double>((ctas + slots - 1) / slots);
    const double cost = waves * (tps + 2.0);  // +2: per-CTA pipeline fill and merge
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = ns;
    }
  }
  DecodePlan plan;
  plan.nsplit = best;
  plan.tiles_per_split = (nkt + best - 1) / best;
  const int64_t rows = static_cast<int64_t>(p->B) * p->Hq * p->Sq * best;
  plan.part_bytes = static_cast<size_t>(rows) * (p->D + 1) * sizeof(float);
  return plan;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t tc_stats_bytes(const cea_attn_params* p) {
  const int nqt = (p->Sq + tc2::BM - 1) / tc2::BM, nkt = (p->Sk + tc2::BN - 1) / tc2::BN;
  return align256(static_cast<size_t>(p->B) * (nqt + nkt) * sizeof(TileStat)) +
         align256(static_cast<size_t>(p->B) * nqt * sizeof(int2));
}

template <typename K>
void allow_smem(K kernel, int bytes) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// ---------------------------------------------------------------- launches
int launch_empty(const cea_attn_params* p, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(p->B) * p->Sq * p->Hq;
  const int grid = static_cast<int>(std::min<int64_t>(rows, 65535));
  const int out_b = elem_bytes(p->out_dtype);
#define CEA_FILL(UO, LT)                                                                                         \
  fill_empty_kernel<UO, LT><<<grid, 64, 0, s>>>(reinterpret_cast<UO*>(p->out), p->o_stride[0], p->o_stride[1],    \
                                                p->o_stride[2], reinterpret_cast<LT*>(p->lse), p->lse_stride[0], \
                                                p->lse_stride[1], p->lse_stride[2], p->B, p->Sq, p->Hq, p->D)
  if (p->in_dtype == CEA_F64) {
    CEA_FILL(uint64_t, double);
  } else if (out_b == 4) {
    CEA_FILL(uint32_t, float);
  } else {
    CEA_FILL(uint16_t, float);
  }
#undef CEA_FILL
  return cuda_check("fill_empty_kernel");
}

// The kernel's setmaxnreg split draws on the registers it is launched with; a build that gave it fewer would
// leave the softmax warps waiting for registers forever, so refuse to launch it.
int check_launch_regs(const void* kernel, int expected) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, kernel) != cudaSuccess) return cuda_check("cudaFuncGetAttributes");
  if (a.numRegs != expected)
    return fail(CEA_ERR_UNSUPPORTED, "prefill kernel built with %d registers per thread, its register split needs %d",
                a.numRegs, expected);
  return CEA_OK;
}

int launch_tc(const cea_attn_params* p, cudaStream_t s) {
  const size_t need = tc_stats_bytes(p);
  if (p->workspace == nullptr || p->workspace_bytes < need)
    return fail(CEA_ERR_WORKSPACE, "tcgen05 attention needs %zu workspace bytes, got %zu", need, p->workspace_bytes);
  const int nqt = (p->Sq + tc2::BM - 1) / tc2::BM, nkt = (p->Sk + tc2::BN - 1) / tc2::BN;
  TileStat* qstat = reinterpret_cast<TileStat*>(p->workspace);
  TileStat* kstat = qstat + static_cast<size_t>(p->B) * nqt;
  int2* qrange = reinterpret_cast<int2*>(reinterpret_cast<uint8_t*>(p->workspace) +
                                         align256(static_cast<size_t>(p->B) * (nqt + nkt) * sizeof(TileStat)));
  {
    const int wq = p->B * nqt, wk = p->B * nkt;
    tile_stats_kernel<<<(wq + 3) / 4, 128, 0, s>>>(p->q_pos, p->qpos_stride[0], p->qpos_stride[1], p->Sq, nqt, p->B,
                                                   0, qstat);
    tile_stats_kernel<<<(wk + 3) / 4, 128, 0, s>>>(p->k_pos, p->kpos_stride[0], p->kpos_stride[1], p->Sk, nkt, p->B,
                                                   1, kstat);
    tile_range_kernel<<<(wq + 3) / 4, 128, 0, s>>>(qstat, kstat, nqt, nkt, p->B, p->causal, qrange);
    if (int e = cuda_check("tile_stats_kernel")) return e;
  }
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, p->in_dtype, p->q, p->D, p->Sq, p->Hq, p->B, p->q_stride[1], p->q_stride[2], p->q_stride[0], 128) ||
      !make_map(&mk, p->in_dtype, p->k, p->D, p->Sk, p->Hkv, p->B, p->k_stride[1], p->k_stride[2], p->k_stride[0], 128) ||
      !make_map(&mv, p->in_dtype, p->v, p->D, p->Sk, p->Hkv, p->B, p->v_stride[1], p->v_stride[2], p->v_stride[0], 128))
    return fail(CEA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the attention operands");
  tc2::AttnArgs tp;
  tp.q_pos = p->q_pos;
  tp.k_pos = p->k_pos;
  tp.qpos_sb = p->qpos_stride[0];
  tp.qpos_ss = p->qpos_stride[1];
  tp.kpos_sb = p->kpos_stride[0];
  tp.kpos_ss = p->kpos_stride[1];
  tp.out = p->out;
  tp.o_sb = p->o_stride[0];
  tp.o_ss = p->o_stride[1];
  tp.o_sh = p->o_stride[2];
  tp.lse = reinterpret_cast<float*>(p->lse);
  tp.l_sb = p->lse_stride[0];
  tp.l_sh = p->lse_stride[1];
  tp.l_ss = p->lse_stride[2];
  tp.kv_map = p->kv_map;
  tp.qstat = qstat;
  tp.kstat = kstat;
  tp.qrange = qrange;
  tp.B = p->B;
  tp.Sq = p->Sq;
  tp.Sk = p->Sk;
  tp.Hq = p->Hq;
  tp.Hkv = p->Hkv;
  tp.group = p->kv_map ? 1 : p->Hq / p->Hkv;
  tp.nqt = nqt;
  tp.nkt = nkt;
  tp.scale_log2 = static_cast<float>(p->scale * 1.4426950408889634);
  tp.causal = p->causal;
  tp.out_dtype = p->out_dtype;
  tp.accumulate = p->accumulate;
  tp.acc_in = p->acc_in;
  tp.a_sb = p->acc_stride[0];
  tp.a_ss = p->acc_stride[1];
  tp.a_sh = p->acc_stride[2];
  const bool bf = p->in_dtype == CEA_BF16;
  // two query tiles per CTA: a GQA head pair when the uniform grouping pairs heads on one KV head, else two
  // adjacent query tiles of one head (an explicit kv_map lives on the device, so it takes the second form)
  tc2::Params pp;
  pp.base = tp;
  const bool heads_pair = p->kv_map == nullptr && p->Hq % 2 == 0 && (p->Hq / p->Hkv) % 2 == 0;
  pp.pair_heads = heads_pair ? 1 : 0;
  pp.nblk_q = heads_pair ? nqt : (nqt + 1) / 2;
  const int64_t grid2 = static_cast<int64_t>(pp.nblk_q) * p->B * (heads_pair ? p->Hq / 2 : p->Hq);
  if (grid2 > 0x7fffffff) return fail(CEA_ERR_UNSUPPORTED, "grid too large");
#define CEA_TC2(DD, BF)                                                                                        \
  do {                                                                                                         \
    auto k = tc2::attn_fwd_tc2_kernel<DD, BF>;                                                                 \
    if (int e = check_launch_regs(reinterpret_cast<const void*>(k), tc2::kLaunchRegs)) return e;              \
    allow_smem(k, tc2::Layout<DD>::SMEM_ALLOC);                                                                \
    k<<<static_cast<unsigned>(grid2), tc2::NUM_THREADS, tc2::Layout<DD>::SMEM_ALLOC, s>>>(mq, mk, mv, pp);     \
  } while (0)
  if (p->D == 128) {
    if (bf) CEA_TC2(128, true); else CEA_TC2(128, false);
  } else {
    if (bf) CEA_TC2(64, true); else CEA_TC2(64, false);
  }
#undef CEA_TC2
  return cuda_check("attn_fwd_tc2_kernel");
}

int launch_decode_plan(const cea_attn_params* p, cudaStream_t s, const DecodePlan& plan, void* workspace);

int launch_decode(const cea_attn_params* p, cudaStream_t s) {
  const DecodePlan plan = decode_plan(p);
  if (p->workspace == nullptr || p->workspace_bytes < plan.part_bytes)
    return fail(CEA_ERR_WORKSPACE, "split-KV decode needs %zu workspace bytes, got %zu", plan.part_bytes,
                p->workspace_bytes);
  return launch_decode_plan(p, s, plan, p->workspace);
}

// the partials live in `workspace` (plan.part_bytes of it)
int launch_decode_plan(const cea_attn_params* p, cudaStream_t s, const DecodePlan& plan, void* workspace) {
  CUtensorMap mk, mv;
  if (!make_map(&mk, p->in_dtype, p->k, p->D, p->Sk, p->Hkv, p->B, p->k_stride[1], p->k_stride[2], p->k_stride[0],
                dec::BKEYS) ||
      !make_map(&mv, p->in_dtype, p->v, p->D, p->Sk, p->Hkv, p->B, p->v_stride[1], p->v_stride[2], p->v_stride[0],
                dec::BKEYS))
    return fail(CEA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV cache");
  const int64_t rows = static_cast<int64_t>(p->B) * p->Hq * p->Sq;
  dec::Params dp;
  dp.q = p->q;
  dp.q_sb = p->q_stride[0];
  dp.q_ss = p->q_stride[1];
  dp.q_sh = p->q_stride[2];
  dp.q_pos = p->q_pos;
  dp.qpos_sb = p->qpos_stride[0];
  dp.qpos_ss = p->qpos_stride[1];
  dp.k_pos = p->k_pos;
  dp.kpos_sb = p->kpos_stride[0];
  dp.kpos_ss = p->kpos_stride[1];
  dp.part_o = reinterpret_cast<float*>(workspace);
  dp.part_lse = dp.part_o + rows * plan.nsplit * p->D;
  dp.B = p->B;
  dp.Sq = p->Sq;
  dp.Sk = p->Sk;
  dp.Hq = p->Hq;
  dp.Hkv = p->Hkv;
  dp.G = p->Hq / p->Hkv;
  dp.nsplit = plan.nsplit;
  dp.tiles_per_split = plan.tiles_per_split;
  dp.scale_log2 = static_cast<float>(p->scale * 1.4426950408889634);
  dp.causal = p->causal;
  dp.n_new = p->n_new;
  dp.new_k = static_cast<const uint16_t*>(p->new_k);
  dp.new_v = static_cast<const uint16_t*>(p->new_v);
  dp.nk_sb = p->new_k_stride[0];
  dp.nk_ss = p->new_k_stride[1];
  dp.nk_sh = p->new_k_stride[2];
  dp.nv_sb = p->new_v_stride[0];
  dp.nv_ss = p->new_v_stride[1];
  dp.nv_sh = p->new_v_stride[2];
  dp.new_pos = p->new_pos;
  dp.np_sb = p->new_pos_stride[0];
  dp.np_ss = p->new_pos_stride[1];
  // with an append the key views are the caller's (writable) cache
  dp.k = const_cast<uint16_t*>(static_cast<const uint16_t*>(p->k));
  dp.v = const_cast<uint16_t*>(static_cast<const uint16_t*>(p->v));
  dp.k_sb = p->k_stride[0];
  dp.k_ss = p->k_stride[1];
  dp.k_sh = p->k_stride[2];
  dp.v_sb = p->v_stride[0];
  dp.v_ss = p->v_stride[1];
  dp.v_sh = p->v_stride[2];
  dp.k_pos_out = const_cast<int64_t*>(p->k_pos);
  const dim3 grid(plan.nsplit, p->Hkv, p->B);
#define CEA_DEC(DD, BF)                                                                              \
  do {                                                                                               \
    auto k = dec::decode_partial_kernel<DD, BF>;                                                     \
    allow_smem(k, dec::Layout<DD>::SMEM_ALLOC);                                                      \
    k<<<grid, dec::NTHREADS, dec::Layout<DD>::SMEM_ALLOC, s>>>(mk, mv, dp);                          \
  } while (0)
  const bool bf = p->in_dtype == CEA_BF16;
  if (p->D == 128) {
    if (bf) CEA_DEC(128, true); else CEA_DEC(128, false);
  } else {
    if (bf) CEA_DEC(64, true); else CEA_DEC(64, false);
  }
#undef CEA_DEC
  if (int e = cuda_check("decode_partial_kernel")) return e;
  dec::CombineParams cp;
  cp.part_o = dp.part_o;
  cp.part_lse = dp.part_lse;
  cp.out = p->out;
  cp.lse = reinterpret_cast<float*>(p->lse);
  cp.o_sb = p->o_stride[0];
  cp.o_ss = p->o_stride[1];
  cp.o_sh = p->o_stride[2];
  cp.l_sb = p->lse_stride[0];
  cp.l_sh = p->lse_stride[1];
  cp.l_ss = p->lse_stride[2];
  cp.B = p->B;
  cp.Sq = p->Sq;
  cp.Hq = p->Hq;
  cp.D = p->D;
  cp.nsplit = plan.nsplit;
  cp.out_dtype = p->out_dtype;
  cp.accumulate = p->accumulate;
  const int64_t blocks = (rows * 32 + 255) / 256;
  dec::decode_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(cp);
  return cuda_check("decode_combine_kernel");
}

template <typename T, typename A, typename O, int DMAX>
void launch_simt_t(const simt::Params& sp, const cea_attn_params* p, cudaStream_t s) {
  auto k = simt::attn_simt_kernel<T, A, O, DMAX>;
  constexpr size_t bytes = simt::smem_bytes<A, DMAX>();
  allow_smem(k, static_cast<int>(bytes));
  const dim3 grid((p->Sq + simt::BQ - 1) / simt::BQ, p->Hq, p->B);
  k<<<grid, simt::NT, bytes, s>>>(sp);
}

template <typename T, typename A, typename O>
int launch_simt_d(const simt::Params& sp, const cea_attn_params* p, cudaStream_t s) {
  if (p->D <= 32) launch_simt_t<T, A, O, 32>(sp, p, s);
  else if (p->D <= 64) launch_simt_t<T, A, O, 64>(sp, p, s);
  else if (p->D <= 128) launch_simt_t<T, A, O, 128>(sp, p, s);
  else if (sizeof(A) == 4 && p->D <= 256) launch_simt_t<T, A, O, (sizeof(A) == 4 ? 256 : 128)>(sp, p, s);
  else return fail(CEA_ERR_UNSUPPORTED, "head dim %d too large for the CUDA-core attention kernel", p->D);
  return cuda_check("attn_simt_kernel");
}

// the register-tiled fp32 kernel: fp32 in and out, head dim 32 or 64, K/V rows 16-byte aligned (cp.async)
bool f32_ok(const cea_attn_params* p) {
  if (p->in_dtype != CEA_F32 || p->out_dtype != CEA_F32 || (p->D != 32 && p->D != 64)) return false;
  if (!aligned16(p->k) || !aligned16(p->v)) return false;
  for (int i = 0; i < 3; ++i)
    if (p->k_stride[i] % 4 || p->v_stride[i] % 4) return false;
  return true;
}

template <int DD>
int launch_f32(const simt::Params& sp, const cea_attn_params* p, cudaStream_t s) {
  auto k = f32k::attn_f32_kernel<DD>;
  allow_smem(k, static_cast<int>(f32k::Smem<DD>::BYTES));
  const dim3 grid(f32k::grid_x(p->Sq, p->causal != 0), p->Hq, p->B);
  k<<<grid, f32k::NT, f32k::Smem<DD>::BYTES, s>>>(sp);
  return cuda_check("attn_f32_kernel");
}

int launch_simt(const cea_attn_params* p, cudaStream_t s) {
  simt::Params sp;
  sp.q = p->q;
  sp.k = p->k;
  sp.v = p->v;
  sp.out = p->out;
  sp.lse = p->lse;
  sp.q_pos = p->q_pos;
  sp.k_pos = p->k_pos;
  sp.kv_map = p->kv_map;
  sp.q_sb = p->q_stride[0];
  sp.q_ss = p->q_stride[1];
  sp.q_sh = p->q_stride[2];
  sp.k_sb = p->k_stride[0];
  sp.k_ss = p->k_stride[1];
  sp.k_sh = p->k_stride[2];
  sp.v_sb = p->v_stride[0];
  sp.v_ss = p->v_stride[1];
  sp.v_sh = p->v_stride[2];
  sp.o_sb = p->o_stride[0];
  sp.o_ss = p->o_stride[1];
  sp.o_sh = p->o_stride[2];
  sp.l_sb = p->lse_stride[0];
  sp.l_sh = p->lse_stride[1];
  sp.l_ss = p->lse_stride[2];
  sp.qpos_sb = p->qpos_stride[0];
  sp.qpos_ss = p->qpos_stride[1];
  sp.kpos_sb = p->kpos_stride[0];
  sp.kpos_ss = p->kpos_stride[1];
  sp.B = p->B;
  sp.Sq = p->Sq;
  sp.Sk = p->Sk;
  sp.Hq = p->Hq;
  sp.Hkv = p->Hkv;
  sp.D = p->D;
  sp.group = p->kv_map ? 1 : p->Hq / p->Hkv;
  sp.scale = p->scale;
  sp.causal = p->causal;
  sp.accumulate = p->accumulate;
  if (f32_ok(p)) return p->D == 64 ? launch_f32<64>(sp, p, s) : launch_f32<32>(sp, p, s);
  switch (p->in_dtype) {
    case CEA_F64:
      return launch_simt_d<double, double, double>(sp, p, s);
    case CEA_F32:
      return launch_simt_d<float, float, float>(sp, p, s);
    case CEA_BF16:
      return p->out_dtype == CEA_F32 ? launch_simt_d<__nv_bfloat16, float, float>(sp, p, s)
                                     : launch_simt_d<__nv_bfloat16, float, __nv_bfloat16>(sp, p, s);
    case CEA_F16:
      return p->out_dtype == CEA_F32 ? launch_simt_d<__half, float, float>(sp, p, s)
                                     : launch_simt_d<__half, float, __half>(sp, p, s);
  }
  return fail(CEA_ERR_UNSUPPORTED, "dtype");
}

}  // namespace

extern "C" {

const char* cea_last_error(void) { return g_last_error.c_str(); }

int cea_abi_version(void) { return CEA_ABI_VERSION; }

int cea_attn_kernel_kind(const cea_attn_params* p) {
  if (validate(p) != CEA_OK) return -1;
  return select_kind(p);
}

size_t cea_attn_workspace_size(const cea_attn_params* p) {
  if (validate(p) != CEA_OK) return 0;
  switch (select_kind(p)) {
    case kTc:
      return tc_stats_bytes(p);
    case kDecode:
      return align256(decode_plan(p).part_bytes);
    default:
      return 0;
  }
}

int cea_attn_fwd(const cea_attn_params* p, void* stream) {
  if (int e = validate(p)) return e;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->B == 0 || p->Sq == 0 || p->Hq == 0) return CEA_OK;
  if (p->Sk == 0) return p->accumulate ? CEA_OK : launch_empty(p, s);
  const int kind = select_kind(p);
  if (p->n_new > 0 && kind != kDecode)
    return fail(CEA_ERR_UNSUPPORTED, "the fused cache append runs on the split-KV decode path only "
                                     "(cea_attn_kernel_kind 2); append the tokens separately");
  if (p->acc_in != nullptr && kind != kTc)
    return fail(CEA_ERR_UNSUPPORTED, "acc_in runs on the tcgen05 path only (cea_attn_kernel_kind 1): bf16/f16, "
                                     "D in {64,128}, TMA-aligned operands, 16-byte aligned out and acc_in rows");
  switch (kind) {
    case kDecode:
      return launch_decode(p, s);
    case kTc:
      return launch_tc(p, s);
    default:
      return launch_simt(p, s);
  }
}

int cea_decode_splitkv(const cea_attn_params* p, void* stream) {
  if (int e = validate(p)) return e;
  if (p->B == 0 || p->Sq == 0 || p->Hq == 0) return CEA_OK;
  if (p->Sk == 0) return p->accumulate ? CEA_OK : launch_empty(p, reinterpret_cast<cudaStream_t>(stream));
  if (!decode_ok(p))
    return fail(CEA_ERR_UNSUPPORTED,
                "split-KV decode needs bf16/f16, D in {64,128}, uniform GQA, Sq*group <= 16 and TMA-aligned K/V");
  return launch_decode(p, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Split-KV decode for callers that cannot allocate device memory.
//
// The per-split partials live in a file-scope device array instead of a
// caller-provided workspace.  Host code must not use the array's name as a
// device address: its address is obtained once per device, with that device
// current, through cudaGetSymbolAddress, and passed to the kernels.  The array
// is shared by every call on a device, so calls that overlap on the GPU (on
// different streams) race on it.  Nothing in it has to start at zero: every
// partial the combine step reads is written by the same call first.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[CEA_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
struct NoallocSlot {
  void* ctx;  // CUDA context the address was looked up in
  void* ptr;
};
NoallocSlot g_noalloc_slot[kNoallocMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
               ? reinterpret_cast<CtxGetCurrentFn>(ptr)
               : nullptr;
  }();
  return fn;
}

// device address of g_noalloc_scratch in the current context of the current device: looked up on the first
// call there, and again when the context changed (a device reset makes a new primary context, into which
// the module and its array are loaded afresh)
int noalloc_scratch(void** out) {
  int dev = 0;
  const cudaError_t ge = cudaGetDevice(&dev);
  if (ge != cudaSuccess) return fail(CEA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(ge));
  if (dev < 0 || dev >= kNoallocMaxDevices)
    return fail(CEA_ERR_UNSUPPORTED, "device %d is beyond the %d devices the decode scratch table covers", dev,
                kNoallocMaxDevices);
  const CtxGetCurrentFn get = ctx_get_current_fn();
  if (get == nullptr) return fail(CEA_ERR_CUDA, "cuCtxGetCurrent is not available from the CUDA driver");
  auto current = [&]() -> void* {
    CUcontext c = nullptr;
    return get(&c) == CUDA_SUCCESS ? static_cast<void*>(c) : nullptr;
  };
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocSlot& slot = g_noalloc_slot[dev];
  void* ctx = current();  // none before the runtime has initialised this device in this process
  if (ctx == nullptr || slot.ptr == nullptr || slot.ctx != ctx) {
    void* ptr = nullptr;
    // also makes the device's primary context current when no context is yet (the lookup allocates nothing)
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(CEA_ERR_CUDA, "cudaGetSymbolAddress of the decode scratch on device %d: %s", dev,
                  cudaGetErrorString(e));
    slot.ctx = current();
    slot.ptr = ptr;
  }
  *out = slot.ptr;
  return CEA_OK;
}

}  // namespace

extern "C" {

int cea_decode_splitkv_noalloc(const cea_attn_params* p, void* stream) {
  if (int e = validate(p)) return e;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->B == 0 || p->Sq == 0 || p->Hq == 0) return CEA_OK;
  if (p->Sk == 0) return p->accumulate ? CEA_OK : launch_empty(p, s);
  if (!decode_ok(p))
    return fail(CEA_ERR_UNSUPPORTED,
                "split-KV decode needs bf16/f16, D in {64,128}, uniform GQA, Sq*group <= 16 and TMA-aligned K/V");
  const DecodePlan plan = decode_plan(p, CEA_NOALLOC_SCRATCH_BYTES);
  if (plan.nsplit == 0)
    return fail(CEA_ERR_WORKSPACE,
                "allocation-free decode: one split of partials for B*Hq*Sq = %lld rows needs %zu bytes, more than the "
                "fixed %u-byte scratch",
                static_cast<long long>(p->B) * p->Hq * p->Sq, plan.part_bytes,
                static_cast<unsigned>(CEA_NOALLOC_SCRATCH_BYTES));
  void* scratch = nullptr;
  if (int e = noalloc_scratch(&scratch)) return e;
  return launch_decode_plan(p, s, plan, scratch);
}

int cea_merge(const cea_merge_params* p, void* stream) {
  if (p == nullptr || p->n < 1 || p->n > CEA_MAX_MERGE) return fail(CEA_ERR_INVALID, "merge needs 1..%d partials", CEA_MAX_MERGE);
  if (p->B < 0 || p->Sq < 0 || p->H < 0 || p->D < 1) return fail(CEA_ERR_INVALID, "invalid merge sizes");
  if (p->out == nullptr) return fail(CEA_ERR_INVALID, "null merge output");
  for (int i = 0; i < p->n; ++i)
    if (p->outs[i] == nullptr || p->lses[i] == nullptr) return fail(CEA_ERR_INVALID, "null partial %d", i);
  const int64_t rows = static_cast<int64_t>(p->B) * p->Sq * p->H;
  if (rows == 0) return CEA_OK;
  MergeArgs a;
  a.n = p->n;
  for (int i = 0; i < p->n; ++i) {
    a.outs[i] = p->outs[i];
    a.lses[i] = p->lses[i];
  }
  a.out = p->out;
  a.lse = p->lse;
  a.po_sb = p->part_o_stride[0];
  a.po_ss = p->part_o_stride[1];
  a.po_sh = p->part_o_stride[2];
  a.pl_sb = p->part_lse_stride[0];
  a.pl_sh = p->part_lse_stride[1];
  a.pl_ss = p->part_lse_stride[2];
  a.o_sb = p->o_stride[0];
  a.o_ss = p->o_stride[1];
  a.o_sh = p->o_stride[2];
  a.l_sb = p->lse_stride[0];
  a.l_sh = p->lse_stride[1];
  a.l_ss = p->lse_stride[2];
  a.B = p->B;
  a.Sq = p->Sq;
  a.H = p->H;
  a.D = p->D;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = static_cast<unsigned>((rows * 32 + 255) / 256);
  if (p->part_dtype == CEA_F32) {
    if (p->out_dtype == CEA_F32) merge_kernel<float, float><<<blocks, 256, 0, s>>>(a);
    else if (p->out_dtype == CEA_BF16) merge_kernel<float, __nv_bfloat16><<<blocks, 256, 0, s>>>(a);
    else if (p->out_dtype == CEA_F16) merge_kernel<float, __half><<<blocks, 256, 0, s>>>(a);
    else return fail(CEA_ERR_UNSUPPORTED, "merge output dtype %d for fp32 partials", p->out_dtype);
  } else if (p->part_dtype == CEA_F64) {
    if (p->out_dtype == CEA_F64) merge_kernel<double, double><<<blocks, 256, 0, s>>>(a);
    else if (p->out_dtype == CEA_F32) merge_kernel<double, float><<<blocks, 256, 0, s>>>(a);
    else return fail(CEA_ERR_UNSUPPORTED, "merge output dtype %d for fp64 partials", p->out_dtype);
  } else {
    return fail(CEA_ERR_UNSUPPORTED, "merge partial dtype %d", p->part_dtype);
  }
  return cuda_check("merge_kernel");
}

static int copy_segments(const cea_copy_params* p, void* stream, const char* what) {
  if (p == nullptr || p->n < 0 || p->n > CEA_MAX_SEGMENTS) return fail(CEA_ERR_INVALID, "%s: 0..%d segments", what, CEA_MAX_SEGMENTS);
  if (p->elem_bytes != 2 && p->elem_bytes != 4 && p->elem_bytes != 8) return fail(CEA_ERR_INVALID, "%s: element size", what);
  if (p->D < 1) return fail(CEA_ERR_INVALID, "%s: D", what);
  CopyArgs a;
  a.n = p->n;
  a.D = p->D;
  a.elem_bytes = p->elem_bytes;
  bool vec = (static_cast<int64_t>(p->D) * p->elem_bytes) % 16 == 0;
  int64_t most = 0;
  for (int i = 0; i < p->n; ++i) {
    const cea_segment& sg = p->seg[i];
    if (sg.nb < 0 || sg.ns < 0 || sg.nh < 0) return fail(CEA_ERR_INVALID, "%s: segment %d sizes", what, i);
    const int64_t rows = static_cast<int64_t>(sg.nb) * sg.ns * sg.nh;
    if (rows > 0 && (sg.src == nullptr || sg.dst == nullptr)) return fail(CEA_ERR_INVALID, "%s: null segment %d", what, i);
    most = std::max(most, rows);
    vec = vec && aligned16(sg.src) && aligned16(sg.dst);
    for (int j = 0; j < 3; ++j)
      vec = vec && (sg.src_stride[j] * p->elem_bytes) % 16 == 0 && (sg.dst_stride[j] * p->elem_bytes) % 16 == 0;
    a.seg[i] = sg;
  }
  a.vec = vec ? 1 : 0;
  if (p->n == 0 || most == 0) return CEA_OK;
  const int64_t units = vec ? (static_cast<int64_t>(p->D) * p->elem_bytes / 16) : p->D;
  const int64_t blocks = std::min<int64_t>((most * units + 255) / 256, 4 * 148 * 4);
  copy_segments_kernel<<<dim3(static_cast<unsigned>(blocks), p->n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cuda_check(what);
}

int cea_ulysses_pack(const cea_copy_params* p, void* stream) { return copy_segments(p, stream, "cea_ulysses_pack"); }
int cea_ulysses_unpack(const cea_copy_params* p, void* stream) { return copy_segments(p, stream, "cea_ulysses_unpack"); }

}  // extern "C"

namespace {

template <typename I>
int launch_wire_to(const cea::wire::Args& a, int dst_dtype, dim3 grid, cudaStream_t s) {
  switch (dst_dtype) {
    case CEA_F32: cea::wire::wire_cast_kernel<I, float><<<grid, cea::wire::kThreads, 0, s>>>(a); return CEA_OK;
    case CEA_F16: cea::wire::wire_cast_kernel<I, __half><<<grid, cea::wire::kThreads, 0, s>>>(a); return CEA_OK;
    case CEA_BF16: cea::wire::wire_cast_kernel<I, __nv_bfloat16><<<grid, cea::wire::kThreads, 0, s>>>(a); return CEA_OK;
    case CEA_F64: cea::wire::wire_cast_kernel<I, double><<<grid, cea::wire::kThreads, 0, s>>>(a); return CEA_OK;
  }
  return fail(CEA_ERR_UNSUPPORTED, "cea_wire_cast: destination dtype %d", dst_dtype);
}

}  // namespace

extern "C" {

int cea_wire_cast(const cea_wire_cast_params* p, void* stream) {
  const char* what = "cea_wire_cast";
  if (p == nullptr) return fail(CEA_ERR_INVALID, "%s: null params", what);
  if (p->B < 0 || p->S < 0 || p->H < 0 || p->D < 0) return fail(CEA_ERR_INVALID, "%s: negative size", what);
  const auto known = [](int d) { return d == CEA_F32 || d == CEA_F16 || d == CEA_BF16 || d == CEA_F64; };
  if (!known(p->src_dtype) || !known(p->dst_dtype)) return fail(CEA_ERR_UNSUPPORTED, "%s: dtype", what);
  const int64_t elems = static_cast<int64_t>(p->B) * p->S * p->H * p->D;
  if (elems == 0) return CEA_OK;
  for (int t = 0; t < 2; ++t)
    if (p->src[t] == nullptr || p->dst[t] == nullptr) return fail(CEA_ERR_INVALID, "%s: null tensor %d", what, t);
  if (p->src_dtype == p->dst_dtype) {
    // no conversion (the wire is not narrower): the strided segment copy, 16 bytes per access when aligned
    cea_copy_params c{};
    c.n = 2;
    c.D = p->D;
    c.elem_bytes = p->src_dtype == CEA_F64 ? 8 : (p->src_dtype == CEA_F32 ? 4 : 2);
    for (int t = 0; t < 2; ++t) {
      cea_segment& sg = c.seg[t];
      sg.src = p->src[t];
      sg.dst = p->dst[t];
      for (int j = 0; j < 3; ++j) {
        sg.src_stride[j] = p->src_stride[t][j];
        sg.dst_stride[j] = p->dst_stride[t][j];
      }
      sg.nb = p->B;
      sg.ns = p->S;
      sg.nh = p->H;
    }
    return copy_segments(&c, stream, what);
  }
  cea::wire::Args a{};
  for (int t = 0; t < 2; ++t) {
    a.src[t] = p->src[t];
    a.dst[t] = p->dst[t];
    for (int j = 0; j < 3; ++j) {
      a.src_stride[t][j] = p->src_stride[t][j];
      a.dst_stride[t][j] = p->dst_stride[t][j];
    }
  }
  a.B = p->B;
  a.S = p->S;
  a.H = p->H;
  a.D = p->D;
  const int64_t groups = elems / p->D * ((p->D + cea::wire::kVec - 1) / cea::wire::kVec);
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>((groups + cea::wire::kThreads - 1) / cea::wire::kThreads,
                                                          148 * 8)), 2);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = CEA_OK;
  switch (p->src_dtype) {
    case CEA_F32: rc = launch_wire_to<float>(a, p->dst_dtype, grid, s); break;
    case CEA_F16: rc = launch_wire_to<__half>(a, p->dst_dtype, grid, s); break;
    case CEA_BF16: rc = launch_wire_to<__nv_bfloat16>(a, p->dst_dtype, grid, s); break;
    default: rc = launch_wire_to<double>(a, p->dst_dtype, grid, s); break;
  }
  return rc != CEA_OK ? rc : cuda_check(what);
}

int cea_add_rmsnorm(const cea_rmsnorm_params* p, void* stream) {
  const char* what = "cea_add_rmsnorm";
  if (p == nullptr) return fail(CEA_ERR_INVALID, "%s: null params", what);
  if (p->rows < 0 || p->h < 1) return fail(CEA_ERR_INVALID, "%s: rows >= 0 and h >= 1", what);
  if (p->rows == 0) return CEA_OK;
  if (!p->resid || !p->weight || !p->y) return fail(CEA_ERR_INVALID, "%s: null pointer", what);
  if (!(p->eps >= 0.0)) return fail(CEA_ERR_INVALID, "%s: eps", what);
  cea::llama::NormArgs a{p->resid, p->delta, p->weight, p->y, p->rows, p->h,
                         p->resid_stride, p->delta_stride, p->y_stride, p->eps};
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(p->rows, 148 * 16));
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // vectorised form: 16-byte rows that fit in the threads' registers
  const int eb = elem_bytes(p->dtype), n = 16 / eb;
  const bool vec = p->h % n == 0 && p->h <= int64_t(cea::llama::kNormThreads) * cea::llama::kNormMaxVecs * n &&
                   aligned16(p->resid) && aligned16(p->weight) && aligned16(p->y) &&
                   (p->delta == nullptr || aligned16(p->delta)) && p->resid_stride % n == 0 && p->y_stride % n == 0 &&
                   (p->delta == nullptr || p->delta_stride % n == 0);
#define CEA_NORM(T)                                                                              \
  do {                                                                                           \
    if (vec)                                                                                     \
      cea::llama::add_rmsnorm_vec_kernel<T><<<grid, cea::llama::kNormThreads, 0, s>>>(a);        \
    else                                                                                         \
      cea::llama::add_rmsnorm_kernel<T><<<grid, cea::llama::kNormThreads, 0, s>>>(a);            \
  } while (0)
  switch (p->dtype) {
    case CEA_F32: CEA_NORM(float); break;
    case CEA_F16: CEA_NORM(__half); break;
    case CEA_BF16: CEA_NORM(__nv_bfloat16); break;
    case CEA_F64: CEA_NORM(double); break;
    default: return fail(CEA_ERR_UNSUPPORTED, "%s: dtype %d", what, p->dtype);
  }
#undef CEA_NORM
  return cuda_check(what);
}

int cea_rope(const cea_rope_params* p, void* stream) {
  const char* what = "cea_rope";
  if (p == nullptr) return fail(CEA_ERR_INVALID, "%s: null params", what);
  if (p->B < 0 || p->S < 0 || p->Hq < 0 || p->Hk < 0 || p->D < 2 || (p->D & 1))
    return fail(CEA_ERR_INVALID, "%s: sizes (D even and >= 2)", what);
  const int64_t most = static_cast<int64_t>(p->B) * p->S * std::max(p->Hq, p->Hk) * (p->D / 2);
  if (most == 0) return CEA_OK;
  if (!p->pos || !p->inv_freq || (p->Hq && !p->q) || (p->Hk && !p->k)) return fail(CEA_ERR_INVALID, "%s: null pointer", what);
  cea::llama::RopeArgs a{};
  a.x[0] = p->q;
  a.x[1] = p->k;
  for (int j = 0; j < 3; ++j) {
    a.stride[0][j] = p->q_stride[j];
    a.stride[1][j] = p->k_stride[j];
  }
  a.H[0] = p->Hq;
  a.H[1] = p->Hk;
  a.pos = p->pos;
  a.pos_stride[0] = p->pos_stride[0];
  a.pos_stride[1] = p->pos_stride[1];
  a.inv_freq = p->inv_freq;
  a.B = p->B;
  a.S = p->S;
  a.D = p->D;
  // one thread per (token, pair): the token's cos / sin serve every q and k head
  const int64_t pairs = static_cast<int64_t>(p->B) * p->S * (p->D / 2);
  const unsigned grid = static_cast<unsigned>(
      std::min<int64_t>((pairs + cea::llama::kEltThreads - 1) / cea::llama::kEltThreads, 148 * 32));
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (p->dtype) {
    case CEA_F32: cea::llama::rope_token_kernel<float><<<grid, cea::llama::kEltThreads, 0, s>>>(a); break;
    case CEA_F16: cea::llama::rope_token_kernel<__half><<<grid, cea::llama::kEltThreads, 0, s>>>(a); break;
    case CEA_BF16: cea::llama::rope_token_kernel<__nv_bfloat16><<<grid, cea::llama::kEltThreads, 0, s>>>(a); break;
    case CEA_F64: cea::llama::rope_token_kernel<double><<<grid, cea::llama::kEltThreads, 0, s>>>(a); break;
    default: return fail(CEA_ERR_UNSUPPORTED, "%s: dtype %d", what, p->dtype);
  }
  return cuda_check(what);
}

int cea_silu_mul(const cea_silu_mul_params* p, void* stream) {
  const char* what = "cea_silu_mul";
  if (p == nullptr) return fail(CEA_ERR_INVALID, "%s: null params", what);
  if (p->rows < 0 || p->n < 0) return fail(CEA_ERR_INVALID, "%s: sizes", what);
  if (p->rows * p->n == 0) return CEA_OK;
  if (!p->gate || !p->up || !p->out) return fail(CEA_ERR_INVALID, "%s: null pointer", what);
  cea::llama::SiluArgs a{p->gate, p->up, p->out, p->rows, p->n, p->in_stride, p->out_stride};
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int eb = elem_bytes(p->dtype), vn = 16 / eb;
  const bool vec = p->n % vn == 0 && p->in_stride % vn == 0 && p->out_stride % vn == 0 && aligned16(p->gate) &&
                   aligned16(p->up) && aligned16(p->out);
  const unsigned grid = vec ? static_cast<unsigned>(std::min<int64_t>(p->rows, 148 * 16))
                            : static_cast<unsigned>(std::min<int64_t>(
                                  (p->rows * p->n + cea::llama::kEltThreads - 1) / cea::llama::kEltThreads, 148 * 8));
#define CEA_SILU(T)                                                                               \
  do {                                                                                            \
    if (vec)                                                                                      \
      cea::llama::silu_mul_vec_kernel<T><<<grid, cea::llama::kEltThreads, 0, s>>>(a);             \
    else                                                                                          \
      cea::llama::silu_mul_kernel<T><<<grid, cea::llama::kEltThreads, 0, s>>>(a);                 \
  } while (0)
  switch (p->dtype) {
    case CEA_F32: CEA_SILU(float); break;
    case CEA_F16: CEA_SILU(__half); break;
    case CEA_BF16: CEA_SILU(__nv_bfloat16); break;
    case CEA_F64: CEA_SILU(double); break;
    default: return fail(CEA_ERR_UNSUPPORTED, "%s: dtype %d", what, p->dtype);
  }
#undef CEA_SILU
  return cuda_check(what);
}

int cea_kv_append(const cea_kv_append_params* p, void* stream) {
  const char* what = "cea_kv_append";
  if (p == nullptr) return fail(CEA_ERR_INVALID, "%s: null params", what);
  if (p->B < 0 || p->n < 0) return fail(CEA_ERR_INVALID, "%s: B and n must be >= 0", what);
  if (p->Hk < 1 || p->Dk < 1 || p->Hv < 1 || p->Dv < 1) return fail(CEA_ERR_INVALID, "%s: heads and head dims must be >= 1", what);
  if (p->offset < 0 || p->capacity < 0 || p->offset + p->n > p->capacity)
    return fail(CEA_ERR_INVALID, "%s: slots %lld..%lld outside a capacity of %lld", what, (long long)p->offset,
                (long long)(p->offset + p->n), (long long)p->capacity);
  const int eb[2] = {p->k_elem_bytes, p->v_elem_bytes};
  for (int i = 0; i < 2; ++i)
    if (eb[i] != 1 && eb[i] != 2 && eb[i] != 4 && eb[i] != 8) return fail(CEA_ERR_INVALID, "%s: element size %d", what, eb[i]);
  if ((p->pos == nullptr) != (p->pos_cache == nullptr))
    return fail(CEA_ERR_INVALID, "%s: positions need both the source and the cache pointer", what);
  if (static_cast<int64_t>(p->B) * p->n == 0) return CEA_OK;
  if (!p->k || !p->v || !p->k_cache || !p->v_cache) return fail(CEA_ERR_INVALID, "%s: null k/v pointer", what);
  cea::kvc::Args a{};
  const void* src[2] = {p->k, p->v};
  void* dst[2] = {p->k_cache, p->v_cache};
  const int64_t* ss[2] = {p->k_stride, p->v_stride};
  const int64_t* ds[2] = {p->kc_stride, p->vc_stride};
  const int H[2] = {p->Hk, p->Hv}, D[2] = {p->Dk, p->Dv};
  int64_t most = static_cast<int64_t>(p->B) * p->n;
  for (int i = 0; i < 2; ++i) {
    cea::kvc::Tensor& t = a.t[i];
    t.src = static_cast<const uint8_t*>(src[i]);
    t.dst = static_cast<uint8_t*>(dst[i]);
    const int64_t row = static_cast<int64_t>(D[i]) * eb[i];
    uint64_t align = reinterpret_cast<uintptr_t>(src[i]) | reinterpret_cast<uintptr_t>(dst[i]) | row;
    for (int j = 0; j < 3; ++j) {
      t.src_stride[j] = ss[i][j] * eb[i];
      t.dst_stride[j] = ds[i][j] * eb[i];
      align |= static_cast<uint64_t>(t.src_stride[j]) | static_cast<uint64_t>(t.dst_stride[j]);
    }
    int unit = 16;
    while (unit > 1 && (align & (unit - 1))) unit >>= 1;
    t.unit = unit;
    const int64_t units = row / unit;
    const int64_t per_b = static_cast<int64_t>(p->n) * H[i] * units;
    if (per_b * p->B >= (int64_t(1) << 31))
      return fail(CEA_ERR_UNSUPPORTED, "%s: %lld copy units in one call (split the append)", what,
                  (long long)(per_b * p->B));
    t.units = cea::kvc::make_fastdiv(static_cast<uint32_t>(units));
    t.H = cea::kvc::make_fastdiv(static_cast<uint32_t>(H[i]));
    t.per_b = cea::kvc::make_fastdiv(static_cast<uint32_t>(per_b));
    t.total = static_cast<uint32_t>(per_b * p->B);
    most = std::max(most, (per_b * p->B + cea::kvc::kUnroll - 1) / cea::kvc::kUnroll);
  }
  a.pos_src = p->pos;
  a.pos_dst = p->pos_cache;
  a.ps_b = p->pos_stride[0];
  a.ps_s = p->pos_stride[1];
  a.pd_b = p->pc_stride[0];
  a.pd_t = p->pc_stride[1];
  a.B = p->B;
  a.n = p->n;
  a.offset = p->offset;
  const int64_t blocks = std::min<int64_t>((most + cea::kvc::kThreads - 1) / cea::kvc::kThreads, 148 * 8);
  cea::kvc::kv_append_kernel<<<dim3(static_cast<unsigned>(blocks), p->pos ? 3 : 2), cea::kvc::kThreads, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cuda_check(what);
}

int cea_device_status(int* status_out, int clear, void* stream) {
  if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return cuda_check("cea_device_status");
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_cea_status, sizeof(int)) != cudaSuccess) return cuda_check("cea_device_status");
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_cea_status, &zero, sizeof(int)) != cudaSuccess) return cuda_check("cea_device_status");
  }
  if (status_out) *status_out = v;
  return CEA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------- NCCL
namespace {

int nccl_fail(const char* what, cea::nccl::Result r) {
  const auto& a = cea::nccl::api();
  return fail(CEA_ERR_NCCL, "%s: %s", what, a.error_string ? a.error_string(r) : "NCCL error");
}

int nccl_ready() {
  const auto& a = cea::nccl::api();
  return a.ok ? CEA_OK : fail(CEA_ERR_NCCL, "%s", a.why.c_str());
}

bool rank_ok(const cea_nccl_comm* c, int r) { return r >= 0 && r < c->nranks; }

}  // namespace

extern "C" {

int cea_nccl_get_unique_id(void* id_out) {
  if (id_out == nullptr) return fail(CEA_ERR_INVALID, "cea_nccl_get_unique_id: null id buffer");
  if (int e = nccl_ready()) return e;
  cea::nccl::UniqueId id;
  if (const auto r = cea::nccl::api().get_unique_id(&id)) return nccl_fail("ncclGetUniqueId", r);
  memcpy(id_out, id.internal, CEA_NCCL_ID_BYTES);
  return CEA_OK;
}

int cea_nccl_comm_init(cea_nccl_comm** comm_out, int rank, int nranks, const void* id) {
  if (comm_out == nullptr || id == nullptr) return fail(CEA_ERR_INVALID, "cea_nccl_comm_init: null argument");
  *comm_out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(CEA_ERR_INVALID, "cea_nccl_comm_init: rank %d out of range for %d ranks", rank, nranks);
  if (int e = nccl_ready()) return e;
  cea::nccl::UniqueId uid;
  memcpy(uid.internal, id, CEA_NCCL_ID_BYTES);
  cea::nccl::Comm nc = nullptr;
  if (const auto r = cea::nccl::api().comm_init_rank(&nc, nranks, uid, rank)) return nccl_fail("ncclCommInitRank", r);
  *comm_out = new cea_nccl_comm{nc, rank, nranks};
  return CEA_OK;
}

int cea_nccl_comm_destroy(cea_nccl_comm* comm) {
  if (comm == nullptr) return CEA_OK;
  const auto r = cea::nccl::api().comm_destroy(comm->comm);
  delete comm;
  return r ? nccl_fail("ncclCommDestroy", r) : CEA_OK;
}

int cea_nccl_abort(cea_nccl_comm* comm) {
  if (comm == nullptr) return CEA_OK;
  const auto r = cea::nccl::api().comm_abort(comm->comm);
  delete comm;
  return r ? nccl_fail("ncclCommAbort", r) : CEA_OK;
}

int cea_ring_step(cea_nccl_comm* comm, const void* send, size_t send_bytes, int to, void* recv, size_t recv_bytes,
                  int from, void* stream) {
  if (comm == nullptr) return fail(CEA_ERR_INVALID, "cea_ring_step: null communicator");
  if (!rank_ok(comm, to) || !rank_ok(comm, from))
    return fail(CEA_ERR_INVALID, "cea_ring_step: peer out of range (to %d, from %d, %d ranks)", to, from, comm->nranks);
  if ((send_bytes > 0 && send == nullptr) || (recv_bytes > 0 && recv == nullptr))
    return fail(CEA_ERR_INVALID, "cea_ring_step: null buffer");
  const auto s = static_cast<cudaStream_t>(stream);
  if (to == comm->rank || from == comm->rank) {  // a ring of one: the block stays local
    if (to != from || send_bytes != recv_bytes)
      return fail(CEA_ERR_INVALID, "cea_ring_step: a self transfer needs to == from and equal sizes");
    if (send_bytes > 0 && cudaMemcpyAsync(recv, send, send_bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return cuda_check("cea_ring_step");
    return CEA_OK;
  }
  const auto& a = cea::nccl::api();
  if (int e = nccl_ready()) return e;
  if (const auto r = a.group_start()) return nccl_fail("ncclGroupStart", r);
  cea::nccl::Result r = 0;
  if (send_bytes > 0) r = a.send(send, send_bytes, cea::nccl::kUint8, to, comm->comm, s);
  if (r == 0 && recv_bytes > 0) r = a.recv(recv, recv_bytes, cea::nccl::kUint8, from, comm->comm, s);
  const auto r2 = a.group_end();
  if (r) return nccl_fail("ncclSend/ncclRecv", r);
  return r2 ? nccl_fail("ncclGroupEnd", r2) : CEA_OK;
}

int cea_alltoallv(cea_nccl_comm* comm, const void* send, const size_t* send_bytes, const size_t* send_offsets,
                  void* recv, const size_t* recv_bytes, const size_t* recv_offsets, void* stream) {
  if (comm == nullptr || send_bytes == nullptr || send_offsets == nullptr || recv_bytes == nullptr ||
      recv_offsets == nullptr)
    return fail(CEA_ERR_INVALID, "cea_alltoallv: null argument");
  const int n = comm->nranks, me = comm->rank;
  for (int p = 0; p < n; ++p)
    if ((send_bytes[p] > 0 && send == nullptr) || (recv_bytes[p] > 0 && recv == nullptr))
      return fail(CEA_ERR_INVALID, "cea_alltoallv: null buffer");
  if (send_bytes[me] != recv_bytes[me])
    return fail(CEA_ERR_INVALID, "cea_alltoallv: this rank sends itself %zu bytes but expects %zu", send_bytes[me],
                recv_bytes[me]);
  const auto s = static_cast<cudaStream_t>(stream);
  const auto* sb = static_cast<const uint8_t*>(send);
  auto* rb = static_cast<uint8_t*>(recv);
  if (send_bytes[me] > 0 &&
      cudaMemcpyAsync(rb + recv_offsets[me], sb + send_offsets[me], send_bytes[me], cudaMemcpyDeviceToDevice, s) !=
          cudaSuccess)
    return cuda_check("cea_alltoallv");
  if (n == 1) return CEA_OK;
  const auto& a = cea::nccl::api();
  if (int e = nccl_ready()) return e;
  if (const auto r = a.group_start()) return nccl_fail("ncclGroupStart", r);
  cea::nccl::Result r = 0;
  for (int p = 0; p < n && r == 0; ++p) {
    if (p == me) continue;
    if (send_bytes[p] > 0) r = a.send(sb + send_offsets[p], send_bytes[p], cea::nccl::kUint8, p, comm->comm, s);
    if (r == 0 && recv_bytes[p] > 0) r = a.recv(rb + recv_offsets[p], recv_bytes[p], cea::nccl::kUint8, p, comm->comm, s);
  }
  const auto r2 = a.group_end();
  if (r) return nccl_fail("ncclSend/ncclRecv", r);
  return r2 ? nccl_fail("ncclGroupEnd", r2) : CEA_OK;
}

int cea_allgather(cea_nccl_comm* comm, const void* send, void* recv, size_t bytes, void* stream) {
  if (comm == nullptr) return fail(CEA_ERR_INVALID, "cea_allgather: null communicator");
  if (bytes > 0 && (send == nullptr || recv == nullptr)) return fail(CEA_ERR_INVALID, "cea_allgather: null buffer");
  if (bytes == 0) return CEA_OK;
  const auto s = static_cast<cudaStream_t>(stream);
  if (comm->nranks == 1) {
    if (recv != send && cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return cuda_check("cea_allgather");
    return CEA_OK;
  }
  if (int e = nccl_ready()) return e;
  if (const auto r = cea::nccl::api().all_gather(send, recv, bytes, cea::nccl::kUint8, comm->comm, s))
    return nccl_fail("ncclAllGather", r);
  return CEA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------ peer-memory decode merge
extern "C" {

int cea_peer_merge(const cea_peer_merge_params* p, void* stream) {
  if (p == nullptr || p->n < 1 || p->n > CEA_MAX_PEERS || p->rank < 0 || p->rank >= p->n)
    return fail(CEA_ERR_INVALID, "cea_peer_merge: need 1..%d ranks and a rank among them", CEA_MAX_PEERS);
  if (p->epoch < 1) return fail(CEA_ERR_INVALID, "cea_peer_merge: calls are numbered from 1");
  if (p->B < 0 || p->Sq < 0 || p->H < 0 || p->D < 1 || p->W <= p->D || p->W % 4 != 0)
    return fail(CEA_ERR_INVALID, "cea_peer_merge: invalid sizes (W must be a multiple of 4 greater than D)");
  if (p->out == nullptr) return fail(CEA_ERR_INVALID, "cea_peer_merge: null output");
  if (p->out_dtype != CEA_F32 && p->out_dtype != CEA_BF16 && p->out_dtype != CEA_F16)
    return fail(CEA_ERR_UNSUPPORTED, "cea_peer_merge: output dtype must be F32, BF16 or F16");
  for (int q = 0; q < p->n; ++q)
    if (p->bufs[q] == nullptr || p->flags[q] == nullptr || !aligned16(p->bufs[q]) ||
        (reinterpret_cast<uintptr_t>(p->flags[q]) & 7u) != 0)
      return fail(CEA_ERR_INVALID, "cea_peer_merge: rank %d's buffer or counters missing or misaligned", q);
  const int64_t rows = static_cast<int64_t>(p->B) * p->Sq * p->H;
  if (rows == 0) return CEA_OK;
  peer::Args a;
  a.n = p->n;
  a.rank = p->rank;
  a.par = static_cast<int>(p->epoch & 1u);
  for (int q = 0; q < CEA_MAX_PEERS; ++q) {
    a.bufs[q] = q < p->n ? p->bufs[q] : nullptr;
    a.flags[q] = q < p->n ? reinterpret_cast<unsigned long long*>(p->flags[q]) : nullptr;
  }
  a.target = static_cast<unsigned long long>(peer::kGrid) * p->epoch;
  a.rows = rows;
  a.W = p->W;
  a.D = p->D;
  a.B = p->B;
  a.Sq = p->Sq;
  a.H = p->H;
  a.out = p->out;
  a.o_sb = p->o_stride[0];
  a.o_ss = p->o_stride[1];
  a.o_sh = p->o_stride[2];
  a.fault_flag = nullptr;
  if (p->fault_flag != nullptr) {
    // the kernel stores into it: accept only memory a kernel can reach (device, managed or pinned host)
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p->fault_flag) != cudaSuccess || attr.devicePointer == nullptr) {
      cudaGetLastError();
      return fail(CEA_ERR_INVALID, "cea_peer_merge: fault_flag is not memory a kernel can write");
    }
    a.fault_flag = static_cast<int*>(attr.devicePointer);
  }
  a.limit_ns = p->wait_limit_ns ? p->wait_limit_ns : static_cast<unsigned long long>(CEA_WAIT_LIMIT_NS);
  const auto s = static_cast<cudaStream_t>(stream);
  if (p->out_dtype == CEA_F32) {
    peer::peer_merge_kernel<float><<<peer::kGrid, peer::kThreads, 0, s>>>(a);
  } else if (p->out_dtype == CEA_BF16) {
    peer::peer_merge_kernel<__nv_bfloat16><<<peer::kGrid, peer::kThreads, 0, s>>>(a);
  } else {
    peer::peer_merge_kernel<__half><<<peer::kGrid, peer::kThreads, 0, s>>>(a);
  }
  return cuda_check("peer_merge_kernel");
}

int cea_ipc_export(const void* ptr, void* handle_out, size_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(CEA_ERR_INVALID, "cea_ipc_export: null argument");
  typedef CUresult (*RangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range = nullptr;
  if (range == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(CEA_ERR_CUDA, "cea_ipc_export: cuMemGetAddressRange unavailable");
    range = reinterpret_cast<RangeFn>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(CEA_ERR_INVALID, "cea_ipc_export: %p is not device memory", ptr);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(CEA_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == CEA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return CEA_OK;
}

int cea_ipc_open(const void* handle, size_t offset, void** ptr_out, void** base_out) {
  if (handle == nullptr || ptr_out == nullptr || base_out == nullptr)
    return fail(CEA_ERR_INVALID, "cea_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(CEA_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *base_out = base;
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return CEA_OK;
}

int cea_ipc_close(void* base) {
  if (base == nullptr) return CEA_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  return e == cudaSuccess ? CEA_OK : fail(CEA_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
}

}  // extern "C"
