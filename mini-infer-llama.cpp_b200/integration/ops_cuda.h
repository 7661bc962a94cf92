// ops_cuda: the B200 backend plugged under mini-infer's own graph executor.
//
// Reference-side integration code: it is compiled together with the
// reference's sources (it includes their headers) and calls the backend only
// through its C-ABI (include/mi_cuda.h). Nothing in the reference changes:
// mi_tensor, the graph builders, gallocr's reserve/plan, mi_kv_cache_init and
// mi_qwen2_forward (src/model_qwen2.cpp:609-688) run as they are. What an
// attached backend replaces is the last step of that forward,
// mi_graph_compute (src/graph.cpp:75-83): instead of the threadpool walking
// g->exec_nodes with a barrier per node (src/threadpool.cpp:171-180), the
// exec nodes are recorded once into a CUDA graph and replayed on the device.
//
// Memory, mirroring the reference's ownership:
//  * gallocr's arena (src/gallocr.cpp:334-357) becomes ONE cudaMalloc of
//    galloc->arena_size bytes; every planned tensor lives at the same offset
//    (device = d_arena + (t->data - galloc->arena)), views at their view
//    offset, so the plan gallocr made for the step is used unchanged;
//  * the GGUF mmap leaves (WEIGHT) are uploaded once at attach: Q8_0
//    matrices repacked into the GEMV's layout, F32 norms and biases as is;
//  * the KV cache (KV) lives in HBM in the reference's layout
//    [head_dim, n_head_kv, n_ctx] per layer (src/model_qwen2.cpp:557-596);
//  * INPUT leaves (the token ids) are copied in before the replay and the
//    OUTPUT leaf (logits) is copied back into its host buffer after it, so
//    mi_qwen2_forward's own memcpy of the logits reads the device result.
#pragma once

#include <cstdint>
#include <string>

#include "graph.h"
#include "model_qwen2.h"

// Counters of the attached backend (for tests and tools).
struct mi_ops_cuda_stats {
  int64_t steps;             // mi_graph_compute calls run on the device
  int64_t nodes;             // exec nodes dispatched to device kernels / copies
  int64_t views_skipped;     // view nodes of g->nodes that moved no data
  int64_t arena_bytes;       // device arena size (== galloc->arena_size)
  int64_t arena_tensors;     // tensor placements resolved into the arena
  int64_t instantiations;    // CUDA graphs instantiated
  int64_t updates;           // replays that updated the previous executable graph in place
  int64_t weight_bytes;      // weight bytes resident in HBM (packed Q8_0 + F32)
};

// Uploads the model's weights, allocates the device KV cache and the device
// arena for `kv` (after mi_kv_cache_init, which reserved gallocr's arena) on
// `device`, and routes every later mi_graph_compute of this process to the
// device. One backend per process (the reference serializes forwards).
// Returns false with *err set when the model has a weight type or shape the
// device kernels do not cover (non-Q8_0 projections) or a CUDA call fails.
bool mi_ops_cuda_attach(mi_qwen2_model* model, mi_kv_cache* kv, int device, std::string* err);

// Frees the device resources; mi_graph_compute runs on the CPU again.
void mi_ops_cuda_detach();

bool mi_ops_cuda_attached();
mi_ops_cuda_stats mi_ops_cuda_get_stats();

// The device executor for one scheduled graph (what mi_graph_compute runs
// while a backend is attached). Aborts with a message on failure, as the
// reference does on runtime errors (its forward has no error return).
void mi_ops_cuda_graph_compute(mi_cgraph* g);
