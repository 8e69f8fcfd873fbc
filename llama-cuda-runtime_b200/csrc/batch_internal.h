// The batch context's chunked prefill as a library-internal routine (not in
// the C ABI): lcr_batch_prefill runs it on the batch's own paged pools, and
// the single-sequence decode context (lcr_prefill) runs it on its own cache
// through a one-slot batch context that it keeps for the purpose.
#pragma once

#include <cuda.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

struct lcr_batch;

namespace lcrb {

// Where the chunk's K/V rows go and attention reads them: per layer l, the
// pools at kpool / vpool + l * layer_elems, the page table at
// table + l * table_layer_stride (pages of page_size positions, pool_pages of
// them), and the pools' row tensor maps (head_dim columns, 16-row boxes) at
// kvmaps[l * kvmap_layer_stride + {0: K, 1: V}]; `limit` positions in all.
// The contiguous cache of one sequence is the case of one page of max_seq
// positions per layer.
struct PrefillKv {
  bf16* kpool;
  bf16* vpool;
  size_t layer_elems;
  const int32_t* table;
  size_t table_layer_stride;
  int page_size;
  int pool_pages;
  const CUtensorMap* kvmaps;
  int kvmap_layer_stride;
  int limit;
};

// Runs `count` prompt tokens (host ids) at positions start .. start + count - 1
// through every layer on the batch's stream, writing their K/V per `kv`, and
// the last row's fp32 logits to `logits` (device, [vocab]). Asynchronous.
int batch_prefill_into(lcr_batch* c, const PrefillKv& kv, const int32_t* tokens, int count, int start,
                       float* logits);
// The tensor map batch_prefill_into expects over a pool of `rows` K or V
// rows of head_dim bf16 each.
int make_prefill_kv_map(CUtensorMap* out, const bf16* pool, int rows, int head_dim);
// The batch's stream and its status check (LCR_OK, or the status of a failed
// device-side check, which is then cleared).
cudaStream_t batch_stream(lcr_batch* c);
int batch_check_status(lcr_batch* c);

}  // namespace lcrb
