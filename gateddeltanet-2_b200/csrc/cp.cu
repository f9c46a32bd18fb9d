#include "chunk_layout.cuh"
extern "C" int gdn2_cp_transition(const gdn2_chunk_args*, float*, void*, size_t, gdn2_stream_t) { return GDN2_ERR_FLAGS; }
extern "C" int gdn2_cp_compose(const float*, int32_t, int64_t, int64_t, int64_t, float*, gdn2_stream_t) { return GDN2_ERR_FLAGS; }
