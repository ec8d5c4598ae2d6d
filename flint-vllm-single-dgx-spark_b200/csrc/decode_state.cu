// Device-side decode bookkeeping, so a whole decode step (and a sequence of them) runs without the host:
// record the sampled token, advance the position / KV length and compute the next KV-cache slot from the block
// table (vLLM's runner does this on the host before each step: slot = block_table[pos / B] * B + pos % B).
#include "common.cuh"
#include "runtime.cuh"

namespace flint {

__global__ void decode_advance_kernel(const int* __restrict__ tokens, int M, int64_t* positions, int* seq_lens, int64_t* slots,
                                      const int* __restrict__ block_tables, int64_t bt_stride, int max_blocks, int block_size,
                                      int* history, int64_t hist_stride, int* step, int max_steps, int* next_tokens) {
  pdl_wait();
  __shared__ int s;
  if (threadIdx.x == 0) s = *step;
  __syncthreads();
  const int m = threadIdx.x;
  if (m < M) {
    const int tok = tokens[m];
    if (history && s < max_steps) history[m * hist_stride + s] = tok;
    if (next_tokens) next_tokens[m] = tok;
    const int64_t pos = positions[m] + 1;
    positions[m] = pos;
    seq_lens[m] = (int)(pos + 1);
    const int64_t blk = pos / block_size;
    slots[m] = blk < max_blocks ? (int64_t)block_tables[m * bt_stride + blk] * block_size + pos % block_size : -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = s + 1;
  pdl_trigger();
}

}  // namespace flint

using namespace flint;

extern "C" int flint_decode_advance(const int32_t* tokens, int64_t M, int64_t* positions, int32_t* seq_lens, int64_t* slots,
                                    const int32_t* block_tables, int64_t bt_stride, int64_t max_blocks, int64_t block_size,
                                    int32_t* history, int64_t hist_stride, int32_t* step, int64_t max_steps,
                                    int32_t* next_tokens, int pdl, void* stream) {
  if (!tokens || !positions || !seq_lens || !slots || !block_tables || !step) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 1024 || block_size < 1 || max_blocks < 1 || bt_stride < max_blocks) return FLINT_ERR_SHAPE;
  return launch(decode_advance_kernel, dim3(1), dim3(((int)M + 31) / 32 * 32), 0, stream, pdl, (const int*)tokens, (int)M,
                positions, (int*)seq_lens, slots, (const int*)block_tables, bt_stride, (int)max_blocks, (int)block_size,
                (int*)history, hist_stride, (int*)step, (int)max_steps, (int*)next_tokens);
}

namespace flint {

__global__ void keys_to_tokens_kernel(const unsigned long long* __restrict__ keys, int M, int* __restrict__ tokens) {
  pdl_wait();
  if ((int)threadIdx.x < M) tokens[threadIdx.x] = (int)argmax_key_index(keys[threadIdx.x]);
  pdl_trigger();
}

}  // namespace flint

extern "C" int flint_argmax_keys_to_tokens(const uint64_t* keys, int64_t M, int32_t* tokens, int pdl, void* stream) {
  using namespace flint;
  if (!keys || !tokens) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 1024) return FLINT_ERR_SHAPE;
  return launch(keys_to_tokens_kernel, dim3(1), dim3((unsigned)((M + 31) / 32 * 32)), 0, stream, pdl,
                reinterpret_cast<const unsigned long long*>(keys), (int)M, (int*)tokens);
}
