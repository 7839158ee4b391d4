// Host interface of the persistent decode step (decode_persistent.cu).
#pragma once

#include <vector>

#include "common.cuh"

namespace glacier {

// What the persistent step reads from an uploaded model (all device pointers).
struct PersistModel {
  int L = 0, D = 0, F = 0, H = 0, Hkv = 0, hd = 0, V = 0, positions = 0, emb_f32 = 0;
  float eps = 1e-6f;
  std::vector<const Int4Weight*> w;  // qkv, o, gate_up, down per layer, then the LM head
  std::vector<const float*> bqkv, in_norm, post_norm;
  const float* final_norm = nullptr;
  const void* embedding = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
};

struct PersistState;

// Builds the step for `max_lanes` lanes; GLACIER_CUDA_EUNSUPPORTED when the model or
// lane count is outside its contract (the multi-kernel step runs instead).
int persist_create(const PersistModel& pm, size_t max_lanes, size_t max_pages, PersistState** out);
void persist_destroy(PersistState* s);
// One greedy decode step, eligible argmax included; logits_out (may be null: no
// logits are written) receives [lanes, V].
int persist_step(PersistState* st, size_t lanes, const int32_t* tokens, const int32_t* positions,
                 const int32_t* block_tables, size_t max_pages, float* pool, size_t page_floats, bool profile,
                 const uint64_t* eligible, size_t eligible_words, int32_t* tokens_out, int32_t* status_out,
                 float* logits_out, cudaStream_t stream);
// Accumulated device time (ns) and count of each phase of profiled steps since
// the last read: [0] norm + qkv, [1] attention, [2] o, [3] norm + gate/up,
// [4] SwiGLU + down, [5] final norm + LM head, [6] logits and the argmax.
int persist_read_stats(PersistState* st, unsigned long long* ns, unsigned long long* n);
int persist_device_error(int clear);

}  // namespace glacier
