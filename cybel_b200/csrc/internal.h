// Internal host-side interfaces shared by the .cu files of libb200q.so.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/b200q.h"

namespace b200q {

struct FmtInfo {
    int elems;            // elements per block
    int bytes;            // bytes per block
    int lanes_per_block;  // GEMV lanes sharing one block
    int blocks_per_slice; // blocks one GEMV warp covers
    int group;            // elements per integer-sum group
    bool r4;              // 4-row block-major layout
};

bool fmt_info(int qtype, FmtInfo& f);
long long row_bytes_of(int qtype, int k);

// Per-device runtime state owned by the library.
struct Device {
    int id = -1;
    int num_sms = 0;
    volatile int* status_host = nullptr;  // host view of the mapped status word
    volatile int* status = nullptr;       // device view (kernels write STATUS_* values)
};
Device* device_state(int dev, int* err);
int current_device_state(Device** out);

// Launch the decode GEMV for m activation rows (looping over row chunks).
// All pointers are device pointers. Returns a B200Q_* status.
int launch_gemv(int qtype, int act_mode, const void* w, const float* x, float* y, int m, int k, int n,
                long long x_stride, long long y_stride, int32_t* isums, Device* dev, cudaStream_t st, bool pdl,
                int flags = 0);

bool pdl_enabled();
void set_last_error(int status);

}  // namespace b200q
