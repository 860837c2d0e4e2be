// Kernels and layout of the peer-sharded gradient exchange (fg_peer.cu) used
// by the data-parallel MLP step (fg_mlp.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

namespace fg {

constexpr int kMaxPeers = 8;       // ranks of one NVLink domain (one box)
constexpr int kMaxPeerParts = 8;   // row blocks of a layer's dW
// The exchange's waits give up after this many nanoseconds of the global
// timer: long enough for ranks whose hosts enqueue the same step some time
// apart.
constexpr unsigned long long kPeerWaitNs = 10ull * 1000 * 1000 * 1000;

// One gradient chunk: [off, off + len) floats of the gradient area, split
// into nranks shards of len / nranks floats (shard r is owned by rank r).
struct PeerChunk {
  size_t off = 0, len = 0;
  int layer = 0, part = 0;
};

// A rank's exchange region, in floats:
//   [grad G | stage G | P0 G | P1 G | LO0 G | LO1 G | flags]
// grad: this rank's gradients (the owned shard of each chunk is overwritten
// by the reduced gradient); stage: peers' contributions to the owned shards
// (chunk c, sender j at c.off + j * shard); P0/P1: parameters of even/odd
// steps in the gradient layout (the loss slot of layer 0's bucket carries
// the global loss); LO0/LO1: TF32 residuals of P0/P1; flags: uint32 words,
// reduce-scatter flags [chunk][sender] then all-gather flags.
struct PeerLayout {
  int nranks = 0, parts = 1;
  size_t grad = 0;               // G
  std::vector<size_t> w_off, b_off;
  size_t loss_off = 0;
  std::vector<PeerChunk> chunks;  // in backward order (the exchange order)
  std::vector<int> first_chunk, n_chunks;  // per layer
  size_t flag_words = 0;
  size_t region = 0;              // floats
  uint32_t digest = 0;            // of everything above (handles must agree)
};

// Host-only.  Returns 0 or an FG_ERR_* code (error message set).
int peer_layout(int n_layers, const int *dims, int nranks, int parts, PeerLayout *out);
// Whether a layer [out, in] can take `parts` dW row blocks.
bool peer_parts_ok(int out, int in, int nranks, int parts);

struct PeerFlagPtrs {
  unsigned int *p[kMaxPeers];  // one flag word in each peer's region (null: none)
};

// Sets each non-null flag word to `val` (release at system scope) once the
// copies ordered before this launch on its stream have completed.
int launch_peer_signal(const PeerFlagPtrs &ptrs, unsigned int val, cudaStream_t st);
// Owned shard of one chunk: a one-block kernel waits (bounded) until
// flags[j] == val for every sender j != rank, then a second kernel sums the
// nranks contributions in rank order and writes the
// sum over the owned shard of `grad`, and the SGD update p_next = p_cur +
// (-(g*lr)) and its TF32 residual over the owned shard; the element at
// loss_idx (chunk-relative, or -1) takes the summed value instead.  All
// pointers are the chunk's base in their area.
// If the wait gives up (after wait_ns of the global timer) it sets the error
// word and the second kernel writes nothing.
int launch_peer_reduce_sgd(float *grad, const float *stage, const float *p_cur, float *p_next,
                           float *lo_next, size_t shard, int rank, int nranks, float lr,
                           long long loss_idx, const unsigned int *flags, unsigned int val,
                           unsigned int *err, int blocks, cudaStream_t st,
                           unsigned long long wait_ns = kPeerWaitNs);
// lo[i] = TF32 residual of p[i] (n a multiple of 4), on at most `blocks` blocks.
int launch_peer_lo(const float *p, float *lo, size_t n, int blocks, cudaStream_t st);
// Waits (bounded) until flags[c * kMaxPeers + j] == val for every chunk c <
// n_chunks and every j < nranks, j != rank.
int launch_peer_wait(const unsigned int *flags, int n_chunks, int nranks, int rank,
                     unsigned int val, unsigned int *err, cudaStream_t st,
                     unsigned long long wait_ns = kPeerWaitNs);

}  // namespace fg
