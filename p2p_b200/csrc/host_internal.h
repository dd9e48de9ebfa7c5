// host_internal.h -- host helpers of api.cu shared with other translation units of the library.
#pragma once

#include <cuda_runtime.h>

#include "../../include/p2p_attn.h"
#include "kernels.h"

namespace p2p {

int ctx_device(const p2p_ctx* ctx);
int ctx_num_sms(const p2p_ctx* ctx);
// Records `msg` as the context's last error and returns `s`.
p2p_status ctx_fail(p2p_ctx* ctx, p2p_status s, const char* msg);
// The shared validation of p2p_attn_params (f32 storage allowed).
p2p_status ctx_check_params(p2p_ctx* ctx, const p2p_attn_params* prm);
float eff_scale_log2(const p2p_attn_params* prm);  // scale (0 -> 1/sqrt(D)) times log2(e)
float eff_eps_of(const p2p_attn_params* prm);      // RMSNorm epsilon (0 -> 1e-5)
int forced_decode_splits();                 // P2P_DECODE_SPLITS (0: not set)
// Device allocations of the library (they honour p2p_debug_set_alloc_limit).
cudaError_t lib_alloc(void** p, size_t bytes);
void lib_free(void* p, size_t bytes);
int32_t* ctx_dev_err(const p2p_ctx* ctx);  // the device error word p2p_sync reports
int32_t debug_wait_deficit();               // p2p_debug_set_wait_deficit's current value

// Argument checks shared by the ragged decode entry points (`who` prefixes the message).
p2p_status check_ragged(p2p_ctx* ctx, const p2p_attn_params* prm, const void* qkv,
                        int64_t ld_qkv, const void* rope, const void* k_cache,
                        const void* v_cache, int64_t kv_rows, const int32_t* offsets,
                        const int32_t* past, int32_t nseq, int32_t max_past, int32_t fused_prep,
                        const void* out, int64_t ld_o, const char* who);
// The ragged-mode fields of DecodeArgs.
void fill_ragged(DecodeArgs& a, const void* qkv, int64_t ld_qkv, const void* norm_w,
                 const void* rope, void* k_cache, void* v_cache, int64_t kv_rows,
                 const int32_t* offsets, const int32_t* past, int32_t max_past, void* out,
                 int64_t ld_o);

// noalloc.cu: looks up the fixed scratch array's device address on `device` (loading the
// module that holds it), so that later no-alloc calls allocate nothing.
cudaError_t noalloc_prepare(int device);

}  // namespace p2p
