// Host launcher of the batched tensor-pipe decode attention (attn_batch.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "attn_batch.cuh"

namespace lcrb {

// Persistent CTAs of attn_batch_launch for a head_dim / group and up to
// `seqs` sequences on `sms` SMs (as many as fit at once).
int attn_batch_ctas(int head_dim, int group, int seqs, int sms, int* ctas);
// One layer's attention for a.seqs sequences (at most kAbMaxSeqs), two
// programmatic launches (attention, then the merge of split partials): kmap /
// vmap = make_kmajor_map of the layer's K / V pool as [pool_pages *
// kv_heads * page_size][head_dim] rows with a {64, 16, head_dim / 64} box;
// `a` as for attn_launch in FUSED paged mode (page_size a multiple of 16),
// plus item_pos (positions per work item, a multiple of 16), a.splits = the
// partial slots per head (at least ceil(max_seq / item_pos), at most
// kAbMaxSplits) and a.work
// (two counters, zero before the first launch; every launch leaves them
// zero).
int attn_batch_launch(const AttnArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int head_dim,
                      int group, int ctas, cudaStream_t s);

}  // namespace lcrb
