// Per-device streams and pooled call workspaces shared by the queued entry points of this library
// (the WNR3 helper batches in helper_abi.cpp and the WNR4 tickets in wnr4_abi.cpp).
#pragma once
#include <cuda_runtime.h>

#include "bufs.h"

namespace wexb {

// The device's upload stream and the kernel stream for a new call (device current): every call's
// record uploads go in call order on the one upload stream, its kernels and read-back on the next of
// four kernel streams, so the kernels of consecutive queued calls may overlap. `meta` (optional): the
// device's stream for launch metadata, so that a call's small metadata copy need not queue behind the
// records of the calls before it. Created once per device and never destroyed (CUDA cannot be called
// while the process unloads). False on a CUDA failure.
bool device_streams(int device, cudaStream_t *up, cudaStream_t *st, cudaStream_t *meta = nullptr);
// The next of the device's 24 hash lanes (a stream and an event to record after its launch): one lane
// per window of verified calls in flight, so that up to 24 windows (1,536 records) hash at once. False
// on a CUDA failure.
bool hash_lane(int device, cudaStream_t *hs, cudaEvent_t *hashed);

// A call's workspace: three events and grown buffers (records, decode scratch, metadata on the device;
// the metadata's page-locked host image). Pooled per device and never freed, like the reference
// helper's pools (c/tools/wex_cuda_bridge.cu:111-153); a queued call holds its workspace until it is
// waited for.
struct Workspace {
    int device = -1;
    cudaEvent_t meta_done = nullptr, uploads_done = nullptr, done = nullptr;
    DevBuf drec, dscratch, dmeta;
    PinBuf hmeta;
    // Upload flags: one device word per record of a call, set by the upload stream after the record's
    // bytes to the call's token, copied from `htoken` (page-locked). Tokens rise by one per call of this
    // workspace, so a word still holding an earlier call's token never reads as landed and the words
    // need no clearing between calls. take_token() returns the next token, or 0 on a CUDA failure; the
    // workspace must be idle. New words are zeroed on stream s first (a bounded wait).
    DevBuf dflags;
    PinBuf htoken;
    uint32_t token = 0;
    uint32_t take_token(size_t records, cudaStream_t s);
};
// A free workspace of `device` (device current), or nullptr on a CUDA / memory failure.
Workspace *workspace_take(int device);
// Returns a workspace to its device's pool. `settled`: everything queued on it has completed; an
// unsettled workspace (its call gave up waiting) is parked and handed out again only once its `done`
// event has completed.
void workspace_give(Workspace *w, bool settled);

}  // namespace wexb
