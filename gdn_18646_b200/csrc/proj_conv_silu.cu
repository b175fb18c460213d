// proj_conv_silu.cu -- fused input projection + causal depthwise conv1d + SiLU.
#include "common.cuh"

namespace gdn {
int check_proj_args(const void* x, const void* W, const void* conv_w, void* y, int B, int T, int D, int Dout,
                    const void* csi, const void* cso, int l2) {
    if (!x || !W || !conv_w || !y) return fail(GDN_ERR_NULL, "gdn_proj_conv_silu_fwd: x, W, conv_w and y are required");
    if (B <= 0 || T <= 0 || D <= 0 || Dout <= 0 || D % 64 != 0 || Dout % 128 != 0)
        return fail(GDN_ERR_SHAPE, "gdn_proj_conv_silu_fwd: need B, T > 0, D %% 64 == 0 and Dout %% 128 == 0 (got B=%d T=%d D=%d Dout=%d)",
                    B, T, D, Dout);
    if (l2 != 0 && (l2 < 8 || l2 > 256 || Dout % l2 != 0 || 128 % l2 != 0))
        return fail(GDN_ERR_SHAPE, "gdn_proj_conv_silu_fwd: l2norm_group %d must divide 128 and Dout", l2);
    if (!aligned16(x) || !aligned16(W) || !aligned16(y) || (reinterpret_cast<uintptr_t>(conv_w) & 7u) ||
        (csi && (reinterpret_cast<uintptr_t>(csi) & 1u)) || (cso && (reinterpret_cast<uintptr_t>(cso) & 1u)))
        return fail(GDN_ERR_ALIGN, "gdn_proj_conv_silu_fwd: x, W, y must be 16-byte and conv_w 8-byte aligned");
    return GDN_OK;
}
}  // namespace gdn

extern "C" int gdn_proj_conv_silu_fwd(const void* x, const void* W, const void* conv_w, void* y, int B, int T,
                                      int D, int Dout, const void* conv_state_in, void* conv_state_out,
                                      int l2norm_group, void* stream) {
    using namespace gdn;
    (void)stream;
    int st = check_proj_args(x, W, conv_w, y, B, T, D, Dout, conv_state_in, conv_state_out, l2norm_group);
    if (st != GDN_OK) return st;
    return fail(GDN_ERR_UNSUPPORTED, "gdn_proj_conv_silu_fwd: not built yet");
}
