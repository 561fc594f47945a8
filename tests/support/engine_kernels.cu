// Test support (not product code): C launchers for the drop-in kernels around the attention path
// — quantised GEMV / GEMM, embedding, add-RMSNorm, argmax, MoE decode and prefill — with the launch
// configurations the reference engine uses (src/engine/weights.hip:239-327, model.hip:88-142,
// moe.hip:53-127), so the GPU tests can check them against oracle/quant.py. Each returns the
// launch status (cudaGetLastError) as an int.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "kernels/argmax.hpp"
#include "kernels/embed.hpp"
#include "kernels/mixed_gemv.hpp"
#include "kernels/moe_decode.hpp"
#include "kernels/moe_prefill.hpp"
#include "kernels/q4k_gemv.hpp"
#include "kernels/q6k_gemv.hpp"
#include "kernels/qgemm.hpp"
#include "kernels/rmsnorm.hpp"

namespace k = miso::kernels;

namespace {

constexpr int kBlock = 256;

template <k::ActFormat A, unsigned K>
void q4k(const k::Q4kGemvParams& p, int rows, unsigned grid) {
  if (rows == 4)
    k::q4k_gemv_kernel<A, K, kBlock, 4><<<grid, kBlock>>>(p);
  else
    k::q4k_gemv_kernel<A, K, kBlock, 1><<<grid, kBlock>>>(p);
}

}  // namespace

extern "C" {

// Q4_K r1 GEMV. rows / grid 0: the engine's choice for FP16 activations (weights.hip:256-267);
// otherwise as given. int8: the per-32 INT8 activation format.
int tk_q4k_gemv(const void* w, const float* x, float* y, unsigned n, unsigned kdim, int int8,
                int rows, unsigned grid) {
  if (rows == 0) {
    rows = (kdim == 2048 && n < 2048) ? 1 : 4;
    grid = rows == 1 ? std::min(240u, std::max(60u, (n + 3) / 4)) : 240u;
  }
  const k::Q4kGemvParams p{static_cast<const std::uint8_t*>(w), x, y, n};
  if (int8) {
    if (kdim == 2048) q4k<k::ActFormat::Int8, 2048>(p, rows, grid);
    else if (kdim == 4096) q4k<k::ActFormat::Int8, 4096>(p, rows, grid);
    else if (kdim == 8192) q4k<k::ActFormat::Int8, 8192>(p, rows, grid);
    else return static_cast<int>(cudaErrorInvalidValue);
  } else {
    if (kdim == 2048) q4k<k::ActFormat::Fp16, 2048>(p, rows, grid);
    else if (kdim == 4096) q4k<k::ActFormat::Fp16, 4096>(p, rows, grid);
    else if (kdim == 8192) q4k<k::ActFormat::Fp16, 8192>(p, rows, grid);
    else return static_cast<int>(cudaErrorInvalidValue);
  }
  return static_cast<int>(cudaGetLastError());
}

// Q6_K r1 GEMV, K = 2048 or 4096. rows / grid 0: the engine's choice (weights.hip:268-279).
int tk_q6k_gemv(const void* w, const float* x, float* y, unsigned n, unsigned kdim, int rows,
                unsigned grid) {
  if (rows == 0) {
    rows = (n >= 8192 && n < 100000) ? 2 : 1;
    grid = rows == 2 ? 480u : (n >= 100000 ? 1920u : 240u);
  }
  const k::Q6kGemvParams p{static_cast<const std::uint8_t*>(w), x, y, n};
  if (kdim == 2048) {
    if (rows == 2) k::q6k_gemv_kernel<2048, kBlock, 2><<<grid, kBlock>>>(p);
    else k::q6k_gemv_kernel<2048, kBlock, 1><<<grid, kBlock>>>(p);
  } else if (kdim == 4096) {
    k::q6k_gemv_kernel<4096, kBlock, 1><<<grid, kBlock>>>(p);
  } else {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return static_cast<int>(cudaGetLastError());
}

// The engine's fused pair (weights.hip:293-299): wide = the q6.n >= 8192 variant.
int tk_mixed_gemv(const void* w6, const void* w4, const float* x, float* y6, float* y4,
                  unsigned n6, unsigned n4, int wide) {
  const k::Q6kGemvParams p6{static_cast<const std::uint8_t*>(w6), x, y6, n6};
  const k::Q4kGemvParams p4{static_cast<const std::uint8_t*>(w4), x, y4, n4};
  if (wide)
    k::mixed_gemv_kernel<2, 480, 240><<<720, kBlock>>>(p6, p4);
  else
    k::mixed_gemv_kernel<1, 240, 240><<<480, kBlock>>>(p6, p4);
  return static_cast<int>(cudaGetLastError());
}

int tk_qgemm_act(const float* x, void* xh, float* xs, unsigned kdim, unsigned n_tok) {
  const k::QGemmActParams p{x, static_cast<__half*>(xh), xs, kdim, n_tok};
  const unsigned groups = n_tok * (kdim / 32);
  k::qgemm_act_kernel<<<(groups + kBlock - 1) / kBlock, kBlock>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int tk_qgemm(int q6, const void* w, const void* xh, const float* xs, float* y, unsigned kdim,
             unsigned n, unsigned n_tok, unsigned ldy) {
  const k::QGemmParams p{static_cast<const std::uint8_t*>(w), static_cast<const __half*>(xh), xs, y,
                         kdim, n, n_tok, ldy};
  const unsigned grid = k::qgemm_tiles(n, n_tok);
  if (q6)
    k::qgemm_kernel<k::QFormat::Q6K><<<grid, kBlock>>>(p);
  else
    k::qgemm_kernel<k::QFormat::Q4K><<<grid, kBlock>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int tk_embed(const void* table, const int* ids, float* out, unsigned tokens) {
  const k::EmbedParams p{static_cast<const std::uint8_t*>(table), ids, out};
  k::embed_q4k_kernel<2048, kBlock><<<tokens, kBlock>>>(p, tokens);
  return static_cast<int>(cudaGetLastError());
}

int tk_add_rmsnorm(float* res, const float* delta, const float* w, float* out, float eps,
                   unsigned tokens, unsigned grid) {
  const k::AddRmsNormParams p{res, delta, w, out, eps};
  k::add_rmsnorm_kernel<2048, k::kRmsNormBlock><<<grid, k::kRmsNormBlock>>>(p, tokens);
  return static_cast<int>(cudaGetLastError());
}

int tk_argmax(const float* x, unsigned n, float* part_v, int* part_i, unsigned parts, int* out) {
  const k::ArgmaxParams p{x, n, part_v, part_i, parts, out};
  k::argmax_partial_kernel<kBlock><<<parts, kBlock>>>(p);
  k::argmax_final_kernel<kBlock><<<1, kBlock>>>(p);
  return static_cast<int>(cudaGetLastError());
}

// One token through the three decode MoE launches (moe.hip:56-79).
int tk_moe_decode(int down_q6, const std::uint16_t* router, const float* x, float* logits,
                  const void* gate_exps, const void* up_exps, const void* gate_sh,
                  const void* up_sh, const void* down_exps, const void* down_sh, float* h,
                  int* ids, float* weights, float* out) {
  using u8 = const std::uint8_t*;
  const k::MoeRouterParams rp{router, x, logits};
  k::moe_router_kernel<kBlock><<<(257 + 3) / 4, kBlock>>>(rp);
  const k::MoeGateUpParams gp{logits, static_cast<u8>(gate_exps), static_cast<u8>(up_exps),
                              static_cast<u8>(gate_sh), static_cast<u8>(up_sh), x, h, ids, weights};
  k::moe_gate_up_kernel<kBlock><<<120, kBlock>>>(gp);
  const k::MoeDownParams dp{logits, ids, weights, static_cast<u8>(down_exps),
                            static_cast<u8>(down_sh), h, out};
  if (down_q6)
    k::moe_down_kernel<k::QType::Q6K, kBlock><<<120, kBlock>>>(dp);
  else
    k::moe_down_kernel<k::QType::Q4K, kBlock><<<120, kBlock>>>(dp);
  return static_cast<int>(cudaGetLastError());
}

unsigned tk_moe_max_tasks(unsigned n) { return k::moe_max_tasks(n); }

// n tokens through the prefill MoE launches (moe.hip:95-127). Scratch sizes as the engine's
// MoePrefillScratch (moe.hip:82-93): xh [n][2048] half, xs [n][64], logits [n][257],
// weights / ids / order [9n], as [9n][32], part [9n][2048], ah [9n][512] half, tasks
// [moe_max_tasks(n)] int4, n_tasks [1].
int tk_moe_prefill(int down_q6, const std::uint16_t* router, const float* x, unsigned n,
                   const void* gate_exps, const void* up_exps, const void* gate_sh,
                   const void* up_sh, const void* down_exps, const void* down_sh, void* xh,
                   float* xs, float* logits, float* weights, int* ids, int* order, int* n_tasks,
                   void* tasks, void* ah, float* as, float* part, float* out) {
  using u8 = const std::uint8_t*;
  const k::QGemmActParams ap{x, static_cast<__half*>(xh), xs, 2048, n};
  k::qgemm_act_kernel<<<(n * 64 + kBlock - 1) / kBlock, kBlock>>>(ap);
  const k::MoeRouterBatchParams rp{router, x, logits, n};
  k::moe_router_batch_kernel<kBlock><<<k::moe_router_batch_items(n, kBlock), kBlock>>>(rp);
  const k::MoeTopkBatchParams tp{logits, ids, weights, n};
  k::moe_topk_batch_kernel<kBlock><<<n, kBlock>>>(tp);
  int4* tk4 = static_cast<int4*>(tasks);
  const k::MoeGroupParams gp{ids, order, tk4, n_tasks, n};
  k::moe_group_kernel<1024><<<1, 1024>>>(gp);
  const unsigned max_tasks = k::moe_max_tasks(n);
  const k::MoeGateUpGroupedParams up{static_cast<u8>(gate_exps), static_cast<u8>(up_exps),
                                     static_cast<u8>(gate_sh), static_cast<u8>(up_sh),
                                     static_cast<const __half*>(xh), xs, order, tk4, n_tasks,
                                     static_cast<__half*>(ah), as};
  k::moe_gate_up_grouped_kernel<kBlock><<<2 * max_tasks, kBlock>>>(up);
  const k::MoeDownGroupedParams dp{static_cast<u8>(down_exps), static_cast<u8>(down_sh),
                                   static_cast<const __half*>(ah), as, weights, order, tk4,
                                   n_tasks, part};
  if (down_q6)
    k::moe_down_grouped_kernel<k::QType::Q6K, kBlock><<<8 * max_tasks, kBlock>>>(dp);
  else
    k::moe_down_grouped_kernel<k::QType::Q4K, kBlock><<<8 * max_tasks, kBlock>>>(dp);
  const k::MoeCombineParams cp{part, out, n};
  k::moe_combine_kernel<<<(n * 512 + 255) / 256, 256>>>(cp);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
