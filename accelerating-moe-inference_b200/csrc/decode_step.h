// The fused batch-1 decode step of the toy MoE decoder (decode_step.cu):
// one cooperative launch runs the whole layer stack and the output head for
// a single sequence, with grid-wide barriers between the dependent phases
// instead of about ten kernel boundaries per layer.
#pragma once

#include <cstddef>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace moe {

// One decoder layer's operands, all on the device.
struct StepLayer {
    const float* attn_norm;        // input RMSNorm weight [d]
    const __nv_bfloat16* wqkv;     // [3d][d]: q rows, then k, then v
    const __nv_bfloat16* wo;       // [d][d]
    float* kc;                     // sequence 0's key cache [H][max_seq][HD]
    float* vc;                     // and value cache
    const float* wg;               // router [E][d] (fp32)
    const float* bias;             // router bias [E], or null
    const float* ffn_norm;         // post-attention RMSNorm weight [d]
    const float* ffn_norm_b;       // its bias (zeros) [d]
    float ffn_eps;
    const __nv_bfloat16* w13;      // [E][2 ffp][d]: blocks of kFfBlock gate rows, then up rows
    const __nv_bfloat16* w2;       // [E][d][ffp]
};

struct StepArgs {
    const StepLayer* layers;       // [nl], device
    int nl, d, H, E, k, ffp, V, max_seq, nch;
    int policy;                    // MoeRouterPolicy
    float quantum, tie_eps;        // PHI-policy parameters
    float eps;                     // input and final RMSNorm epsilon
    float scale;                   // 1 / sqrt(head_dim)
    const int* tok;                // [1] the step's token id
    const float* embed;            // [V][d] fp32 (the gather)
    const float* final_norm;       // [d]
    const __nv_bfloat16* head;     // [V][d] (the tied embedding in bf16)
    const float2* rope;            // [max_seq][HD / 2] (cos, sin)
    const int* pos_dev;            // the step's position
    // Workspace, written and read inside one launch.
    float* qkv;                    // [3d]
    float* attn_part;              // [H][nch][HD + 2]
    float* xm;                     // [d] residual after the attention block
    float* logits_e;               // [E] router logits
    float* h;                      // [k][ffp]
    float* part;                   // [ceil(ffp / kDownChunk)][k][d]
    float* logits;                 // [V] output
    unsigned* sync;                // [4]: 64-bit arrival count (words 0-1), abort word (2);
                                   // 16-byte aligned, zeroed at creation and after an error
    int* err;                      // device error flags
};

// Device error flag of a token id outside [0, vocab) (the decoder's gather).
constexpr int kDecErrToken = 1 << 12;

// Threads per CTA of the fused step.
constexpr int kStepThreads = 384;

// Dynamic shared memory of one CTA.
size_t step_fused_smem(int d, int H, int nch);
// CTAs per SM the fused step can keep resident at `smem` (0: it cannot run).
int step_fused_occupancy(int head_dim, size_t smem);
// Launch on `grid` CTAs (at most one per SM) as a cooperative grid.
cudaError_t launch_step_fused(const StepArgs& a, int head_dim, int grid, size_t smem,
                              cudaStream_t s);

}  // namespace moe
