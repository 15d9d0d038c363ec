// ep.cuh -- expert parallelism: the NCCL communicator of the backend (one
// process per GPU) and the combine of the ranks' partial MoE outputs.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

namespace loom {

bool ep_active();
int ep_rank();
int ep_size();
// Collective: true on every rank when every rank passed the same n ints
// (host values; n <= 16), false on every rank otherwise. Synchronises the
// host with one small NCCL exchange on a private stream.
bool ep_agree(const int *vals, int n, std::string &err);
// out[i] = sum over ranks of out[i] (in place), on stream st
int ep_allreduce_sum(float *buf, size_t n, cudaStream_t st, std::string &err);

// All-to-all exchange of variable-sized runs: send[soff[r], soff[r]+scnt[r])
// units go to rank r, recv[roff[r], roff[r]+rcnt[r]) units come from rank r
// (unit = `unit_bytes`; offsets and counts in units, host arrays of ep_size()
// entries). The run to this rank itself is a device copy. One NCCL group of
// point-to-point sends and receives.
int ep_alltoallv(const void *send, const size_t *soff, const size_t *scnt, void *recv, const size_t *roff,
                 const size_t *rcnt, size_t unit_bytes, cudaStream_t st, std::string &err);

// ---- all-to-all expert parallelism (a2a.cu) ----
constexpr int A2A_MAX_RANKS = 64;
// Route-ordered slots [T][n_used] -> destination-ordered send lists:
// send_eid/send_tok [T*n_used], slot_pos [T*n_used] (position of each slot in
// the send order), cnt [world] (slots per destination), send_x [T*n_used][dim].
// cap > 0: fixed-capacity runs of cap entries per destination (send lists of
// world*cap entries, unused ones with expert and token -1).
void launch_a2a_pack(const int *ids, int T, int n_used, int n_expert, int world, int cap, const float *x, int dim,
                     int *send_eid, int *send_tok, int *slot_pos, int *cnt, float *send_x, cudaStream_t st);
void launch_a2a_fill(float *v, int n, float val, cudaStream_t st);
// out[t] = residual[t] + (sum_k gates[t,k] * y_back[slot_pos[t,k]] + y_sh[t])
void launch_a2a_combine(const float *y_back, const int *slot_pos, const float *gates, const float *y_sh,
                        const float *residual, float *out, int T, int n_used, int dim, cudaStream_t st);

}  // namespace loom
