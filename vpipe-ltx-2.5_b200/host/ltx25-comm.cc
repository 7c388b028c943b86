// ltx25-comm.cc -- Comm (see ltx25-comm.h).
#include "ltx25-comm.h"

#include <dlfcn.h>
#include <cuda_bf16.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

namespace ltx25 {

namespace {

struct Nccl {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclReduceScatter) reduce_scatter = nullptr;
  decltype(&ncclCommSplit) comm_split = nullptr;
  bool ok = false;
  std::string why;
};

const Nccl& nccl()
{
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = nullptr;
    for (const char* name : {"libnccl.so.2", "libnccl.so"}) {
      h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
      if (h != nullptr) break;
    }
    if (h == nullptr) {
      const char* e = dlerror();
      n.why = std::string("NCCL not found: ") + (e ? e : "dlopen failed");
      return;
    }
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.send = reinterpret_cast<decltype(n.send)>(dlsym(h, "ncclSend"));
    n.recv = reinterpret_cast<decltype(n.recv)>(dlsym(h, "ncclRecv"));
    n.group_start = reinterpret_cast<decltype(n.group_start)>(dlsym(h, "ncclGroupStart"));
    n.group_end = reinterpret_cast<decltype(n.group_end)>(dlsym(h, "ncclGroupEnd"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.reduce_scatter =
        reinterpret_cast<decltype(n.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    n.comm_split = reinterpret_cast<decltype(n.comm_split)>(dlsym(h, "ncclCommSplit"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce &&
           n.error_string && n.send && n.recv && n.group_start && n.group_end &&
           n.all_gather && n.reduce_scatter;
    if (!n.ok) n.why = "NCCL library lacks a required symbol";
  });
  return n;
}

bool nccl_ok(ncclResult_t r, const char* what, std::string* err)
{
  if (r == ncclSuccess) return true;
  if (err) *err = std::string(what) + ": " + nccl().error_string(r);
  return false;
}

}  // namespace

bool Comm::unique_id(void* out, std::string* err)
{
  const Nccl& n = nccl();
  if (!n.ok) {
    if (err) *err = n.why;
    return false;
  }
  ncclUniqueId id;
  if (!nccl_ok(n.get_unique_id(&id), "ncclGetUniqueId", err)) return false;
  static_assert(sizeof(id) == kIdBytes, "unique id size");
  memcpy(out, &id, sizeof(id));
  return true;
}

Comm::~Comm()
{
  release_buffers_();
  if (_table != nullptr) cudaFree(_table);
  if (_token != nullptr) cudaFree(_token);   // _vote and _hbuf share its allocation
  if (_comm != nullptr && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(_comm));
}

bool Comm::alloc_words_()
{
  // the barrier word, the vote word and the [8][64] handle exchange in one
  // allocation
  void* p = nullptr;
  if (cudaMalloc(&p, 256 + 8 * 64) != cudaSuccess) return false;
  if (cudaMemset(p, 0, 256 + 8 * 64) != cudaSuccess) {
    cudaFree(p);
    return false;
  }
  _token = static_cast<float*>(p);
  _vote = _token + 1;
  _hbuf = static_cast<char*>(p) + 256;
  return true;
}

void Comm::release_buffers_()
{
  for (int r = 0; r < _world && r < 8; ++r) {
    if (_peer[r] == nullptr) continue;
    if (r == _rank)
      cudaFree(_peer[r]);
    else
      cudaIpcCloseMemHandle(_peer[r]);
    _peer[r] = nullptr;
  }
  _share_bytes = 0;
}

bool Comm::share_buffers(size_t bytes, cudaStream_t s, std::string* err)
{
  if (_comm == nullptr || bytes <= _share_bytes) return true;
  if (_world > 8) return true;   // unavailable: the NCCL reduce-scatter stays
  auto cuda = [&](cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    if (err) *err = std::string(what) + ": " + cudaGetErrorString(e);
    return false;
  };
  const ncclComm_t c = static_cast<ncclComm_t>(_comm);
  // Everything issued before (the previous buffers' last readers and
  // writers on every rank) is done once this returns.
  if (_share_bytes > 0 && !(barrier(s, err) && cuda(cudaStreamSynchronize(s), "sync")))
    return false;
  release_buffers_();
  bytes = (bytes + 255) & ~size_t(255);
  // Every rank takes both collectives below whatever happens locally, so
  // that a rank whose allocation or mapping fails cannot leave the others
  // waiting: a failed rank publishes an empty handle, and the ranks then
  // agree (a sum of failures) to use the buffers or none.
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  memset(&h, 0, sizeof h);
  void* mine = nullptr;
  bool local_ok = cudaMalloc(&mine, 2 * bytes) == cudaSuccess;
  if (local_ok) _peer[_rank] = mine;
  local_ok = local_ok && cudaIpcGetMemHandle(&h, mine) == cudaSuccess;
  if (!local_ok) memset(&h, 0, sizeof h);
  std::vector<char> host((size_t)_world * 64);
  if (!(cuda(cudaMemcpy(_hbuf + (size_t)_rank * 64, &h, 64, cudaMemcpyHostToDevice),
             "handle upload") &&
        nccl_ok(nccl().all_gather(_hbuf + (size_t)_rank * 64, _hbuf, 64, ncclInt8, c, s),
                "ncclAllGather(handles)", err) &&
        cuda(cudaStreamSynchronize(s), "sync") &&
        cuda(cudaMemcpy(host.data(), _hbuf, host.size(), cudaMemcpyDeviceToHost),
             "handle download"))) {
    release_buffers_();
    return false;
  }
  for (int r = 0; local_ok && r < _world; ++r) {
    if (r == _rank) continue;
    cudaIpcMemHandle_t hr;
    memcpy(&hr, host.data() + (size_t)r * 64, 64);
    local_ok = cudaIpcOpenMemHandle(&_peer[r], hr, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    if (!local_ok) _peer[r] = nullptr;
  }
  __nv_bfloat16* tbl[16] = {};
  for (int w = 0; local_ok && w < 2; ++w)
    for (int r = 0; r < _world; ++r)
      tbl[w * 8 + r] = static_cast<__nv_bfloat16*>(_peer[r]) + (size_t)w * (bytes / 2);
  local_ok = local_ok && (_table != nullptr || cudaMalloc(&_table, sizeof tbl) == cudaSuccess) &&
             cudaMemcpy(_table, tbl, sizeof tbl, cudaMemcpyHostToDevice) == cudaSuccess;
  cudaGetLastError();   // a failed IPC call above is this rank's vote, not an error
  float fails = local_ok ? 0.0f : 1.0f;
  if (!(cuda(cudaMemcpy(_vote, &fails, sizeof fails, cudaMemcpyHostToDevice), "vote upload") &&
        nccl_ok(nccl().all_reduce(_vote, _vote, 1, ncclFloat32, ncclSum, c, s),
                "ncclAllReduce(vote)", err) &&
        cuda(cudaStreamSynchronize(s), "sync") &&
        cuda(cudaMemcpy(&fails, _vote, sizeof fails, cudaMemcpyDeviceToHost), "vote download"))) {
    release_buffers_();
    return false;
  }
  if (fails > 0.0f) {
    // some rank cannot map its peers (no peer access on this node): every
    // rank drops the buffers and keeps the NCCL reduce-scatter
    release_buffers_();
    return true;
  }
  _share_bytes = bytes;
  return true;
}

bool Comm::barrier(cudaStream_t s, std::string* err) const
{
  if (_comm == nullptr) return true;
  return nccl_ok(nccl().all_reduce(_token, _token, 1, ncclFloat32, ncclSum,
                                   static_cast<ncclComm_t>(_comm), s),
                 "ncclAllReduce(barrier)", err);
}

bool Comm::init(int device, int rank, int world, const void* id, std::string* err)
{
  const Nccl& n = nccl();
  if (!n.ok) {
    if (err) *err = n.why;
    return false;
  }
  if (world < 1 || rank < 0 || rank >= world) {
    if (err) *err = "tp: rank outside [0, world)";
    return false;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    if (err) *err = "tp: cudaSetDevice failed";
    return false;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  if (!nccl_ok(n.comm_init_rank(&c, world, uid, rank), "ncclCommInitRank", err)) return false;
  _comm = c;
  _rank = rank;
  _world = world;
  _device = device;
  if (!alloc_words_()) {
    if (err) *err = "tp: cudaMalloc(communicator words) failed";
    return false;
  }
  return true;
}

bool Comm::allreduce_sum(void* buf, size_t count, int dtype, cudaStream_t s,
                         std::string* err) const
{
  if (_comm == nullptr || count == 0) return true;
  const ncclDataType_t t = dtype == 0 ? ncclFloat32 : ncclBfloat16;
  return nccl_ok(nccl().all_reduce(buf, buf, count, t, ncclSum,
                                   static_cast<ncclComm_t>(_comm), s),
                 "ncclAllReduce", err);
}

bool Comm::split(Comm* out, std::string* err) const
{
  const Nccl& n = nccl();
  if (_comm == nullptr || n.comm_split == nullptr) {
    if (err) *err = "comm split unavailable";
    return false;
  }
  ncclComm_t c = nullptr;
  if (!nccl_ok(n.comm_split(static_cast<ncclComm_t>(_comm), 0, _rank, &c, nullptr),
               "ncclCommSplit", err))
    return false;
  out->_comm = c;
  out->_rank = _rank;
  out->_world = _world;
  out->_device = _device;
  if (!out->alloc_words_()) {
    if (err) *err = "comm split: cudaMalloc(communicator words) failed";
    return false;
  }
  return true;
}

bool Comm::alltoall_bf16(const void* send, void* recv, size_t count, int n, size_t stride,
                         cudaStream_t s, std::string* err) const
{
  if (_comm == nullptr || count == 0) return true;
  const Nccl& nc = nccl();
  const ncclComm_t c = static_cast<ncclComm_t>(_comm);
  const size_t blk = count * 2;   // bytes per peer block
  if (!nccl_ok(nc.group_start(), "ncclGroupStart", err)) return false;
  bool ok = true;
  for (int i = 0; i < n && ok; ++i) {
    const char* sb = static_cast<const char*>(send) + i * stride * 2;
    char* rb = static_cast<char*>(recv) + i * stride * 2;
    for (int p = 0; p < _world && ok; ++p) {
      ok = nccl_ok(nc.send(sb + p * blk, count, ncclBfloat16, p, c, s), "ncclSend", err) &&
           nccl_ok(nc.recv(rb + p * blk, count, ncclBfloat16, p, c, s), "ncclRecv", err);
    }
  }
  const bool ended = nccl_ok(nc.group_end(), "ncclGroupEnd", ok ? err : nullptr);
  return ok && ended;
}

bool Comm::allgather_bf16(const void* send, void* recv, size_t count, cudaStream_t s,
                          std::string* err) const
{
  if (_comm == nullptr || count == 0) return true;
  return nccl_ok(nccl().all_gather(send, recv, count, ncclBfloat16,
                                   static_cast<ncclComm_t>(_comm), s),
                 "ncclAllGather", err);
}

bool Comm::reduce_scatter_bf16(void* buf, size_t count, cudaStream_t s, std::string* err) const
{
  if (_comm == nullptr || count == 0) return true;
  __nv_bfloat16* b = static_cast<__nv_bfloat16*>(buf);
  return nccl_ok(nccl().reduce_scatter(b, b + (size_t)_rank * count, count, ncclBfloat16,
                                       ncclSum, static_cast<ncclComm_t>(_comm), s),
                 "ncclReduceScatter", err);
}

}  // namespace ltx25
