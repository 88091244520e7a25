// NCCL entry points resolved at run time.  The library does not link libnccl:
// single-GPU use never loads it, and under tensor parallelism it reuses the
// libnccl already in the process (e.g. the one a PyTorch host loaded), so two
// NCCL builds never meet in one process.
#pragma once
#include <nccl.h>

namespace fg {

struct NcclApi {
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRank) CommInitRank = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclAllReduce) AllReduce = nullptr;
  decltype(&ncclAllGather) AllGather = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
};

// Loads libnccl on first use; raises FG_ERR_UNAVAILABLE if it cannot.
const NcclApi &nccl();

}  // namespace fg
