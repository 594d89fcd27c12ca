// Chunked-prefill entry points (interim): the chunk op is served by the token
// recurrence until the chunk-64 tensor-core kernel lands in this file.
#include "kda_common.cuh"

extern "C" size_t kda_chunk_workspace_bytes(int32_t num_req, int32_t num_tokens, int32_t num_heads,
                                            int32_t head_dim) {
    (void)num_req; (void)num_tokens; (void)num_heads; (void)head_dim;
    return 0;
}

extern "C" int kda_chunk_launch(const KdaArgs *args, void *workspace, size_t workspace_bytes, void *stream) {
    (void)workspace; (void)workspace_bytes;
    if (args == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    if (args->intermediate != nullptr) return KDA_ERR_INVALID_ARGUMENT;
    return kda_recurrent_launch(args, stream);
}
