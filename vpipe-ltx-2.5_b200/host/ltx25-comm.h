// ltx25-comm.h -- the tensor-parallel communicator: one NCCL communicator per
// context, reached through dlopen so the library has no link-time NCCL
// dependency (a process that already loaded NCCL, e.g. through PyTorch, shares
// that copy).  The reference has no counterpart: it runs on one Apple GPU.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <string>

namespace ltx25 {

class Comm {
public:
  static constexpr int kIdBytes = 128;   // NCCL_UNIQUE_ID_BYTES

  // A fresh rendezvous id (rank 0 makes it; the caller ships it to the
  // other ranks by any channel).
  static bool unique_id(void* out, std::string* err);

  ~Comm();
  // Join the group: every rank calls this with the same id and world.
  bool init(int device, int rank, int world, const void* id, std::string* err);

  // In-place sum over the group on `s`.  dtype: 0 = f32, 1 = bf16.
  bool allreduce_sum(void* buf, size_t count, int dtype, cudaStream_t s,
                     std::string* err) const;
  // bf16 all-to-all: `count` elements to and from every rank; block p of
  // `send` goes to rank p, block p of `recv` comes from rank p.  `n` such
  // exchanges (send + i * stride, recv + i * stride) in one NCCL group.
  bool alltoall_bf16(const void* send, void* recv, size_t count, int n, size_t stride,
                     cudaStream_t s, std::string* err) const;
  // bf16 all-gather: rank r's `count` elements land at recv + r * count
  // (send may be recv + rank * count: in place).
  bool allgather_bf16(const void* send, void* recv, size_t count, cudaStream_t s,
                      std::string* err) const;

  // bf16 reduce-scatter in place: `buf` holds world * count elements on
  // every rank; rank r's block [r * count, (r + 1) * count) ends as the sum
  // of every rank's block r (the other blocks are left undefined).
  bool reduce_scatter_bf16(void* buf, size_t count, cudaStream_t s, std::string* err) const;

  // A second communicator over the same ranks (ncclCommSplit), for
  // collectives issued on another stream.
  bool split(Comm* out, std::string* err) const;

  // Peer-mapped receive buffers for the fused reduce-scatter: every rank
  // allocates two buffers of `bytes` and maps every other rank's through
  // CUDA IPC, so a kernel here can store into any rank's buffers over
  // NVLink.  Collective (every rank, same bytes, same order); a no-op when
  // the buffers are already that large.  When any rank cannot allocate or
  // map them (no peer access, more than 8 ranks) every rank ends without
  // buffers (shared_bytes() == 0) and true; false only when the
  // communicator itself fails.
  bool share_buffers(size_t bytes, cudaStream_t s, std::string* err);
  size_t shared_bytes() const { return _share_bytes; }
  // Which of the two buffers the next fused reduce-scatter uses: they
  // alternate, so a call's writers never meet the previous call's readers
  // (every rank makes the same calls in the same order).
  int next_buffer() const { return _flip ^= 1; }
  // Buffer `which` of every rank (world entries), as a device array.
  __nv_bfloat16* const* peer_table(int which) const { return _table + (size_t)which * 8; }
  // Rank r's buffer `which` (0 or 1), as mapped in this process.
  void* peer_buffer(int r, int which) const
  {
    return static_cast<char*>(_peer[r]) + (size_t)which * _share_bytes;
  }
  // An ordering point for the group on `s`: returns once every rank's work
  // issued on its stream before it has completed (a 4-byte all-reduce).
  bool barrier(cudaStream_t s, std::string* err) const;

  int rank() const { return _rank; }
  int world() const { return _world; }

private:
  void release_buffers_();
  bool alloc_words_();

  void* _comm = nullptr;
  int _rank = 0, _world = 1, _device = -1;
  void* _peer[8] = {};            // [rank]: this rank's own at _peer[_rank]
  size_t _share_bytes = 0;        // bytes of one of the two buffers
  float* _token = nullptr;        // the barrier's 4 bytes
  float* _vote = nullptr;         // share_buffers' agreement word
  char* _hbuf = nullptr;          // share_buffers' [8][64] IPC handle exchange
  __nv_bfloat16** _table = nullptr;   // device [2][8]: every rank's buffers
  mutable int _flip = 1;          // the buffer of the last fused reduce-scatter
};

}  // namespace ltx25
