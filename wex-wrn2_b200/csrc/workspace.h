// Per-device streams and pooled call workspaces shared by the queued entry points of this library
// (the WNR3 helper batches in helper_abi.cpp and the WNR4 tickets in wnr4_abi.cpp).
#pragma once
#include <cuda_runtime.h>

#include "bufs.h"

namespace wexb {

// The device's upload stream and the kernel stream for a new call (device current): every call's
// uploads go in call order on the one upload stream, its kernels and read-back on the next of four
// kernel streams, so the kernels of consecutive queued calls may overlap. Created once per device and
// never destroyed (CUDA cannot be called while the process unloads). False on a CUDA failure.
bool device_streams(int device, cudaStream_t *up, cudaStream_t *st);
// A stream for a verified call's record hashes (the next of 64 per device): a record's SHA-256 is one
// serial chain, so the hashes of every call in flight must run at once. False on a CUDA failure.
bool hash_stream(int device, cudaStream_t *hs);

// A call's workspace: two events and grown buffers (records, decode scratch, metadata on the device;
// the metadata's page-locked host image). Pooled per device and never freed, like the reference
// helper's pools (c/tools/wex_cuda_bridge.cu:111-153); a queued call holds its workspace until it is
// waited for.
struct Workspace {
    int device = -1;
    cudaEvent_t meta_done = nullptr, hashed = nullptr, uploads_done = nullptr, done = nullptr;
    DevBuf drec, dscratch, dmeta;
    PinBuf hmeta;
};
// A free workspace of `device` (device current), or nullptr on a CUDA / memory failure.
Workspace *workspace_take(int device);
// Returns a workspace to its device's pool. `settled`: everything queued on it has completed; an
// unsettled workspace (its call gave up waiting) is parked and handed out again only once its `done`
// event has completed.
void workspace_give(Workspace *w, bool settled);

}  // namespace wexb
