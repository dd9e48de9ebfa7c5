// host_internal.h -- host helpers of api.cu shared with other translation units of the library.
#pragma once

#include "../../include/p2p_attn.h"

namespace p2p {

int ctx_device(const p2p_ctx* ctx);
int ctx_num_sms(const p2p_ctx* ctx);
// Records `msg` as the context's last error and returns `s`.
p2p_status ctx_fail(p2p_ctx* ctx, p2p_status s, const char* msg);
// The shared validation of p2p_attn_params (f32 storage allowed).
p2p_status ctx_check_params(p2p_ctx* ctx, const p2p_attn_params* prm);
float eff_scale_log2(const p2p_attn_params* prm);  // scale (0 -> 1/sqrt(D)) times log2(e)
float eff_eps_of(const p2p_attn_params* prm);      // RMSNorm epsilon (0 -> 1e-5)

}  // namespace p2p
