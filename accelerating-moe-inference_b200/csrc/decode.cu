// Weight-streaming decode path (small T): not yet built.  forward_impl only
// takes it when T <= decode_max_tokens, which defaults to 0.
#include "moe_internal.h"

namespace moe {

cudaError_t launch_decode(Layer&, const float*, int, float*, cudaStream_t) {
    return cudaErrorNotSupported;
}

}  // namespace moe
