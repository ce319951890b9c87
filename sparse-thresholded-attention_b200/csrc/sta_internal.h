// Internal launch helpers shared by the translation units of libsta.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/sta.h"

namespace sta {

void set_error(const char* msg);
int fail(int code, const char* msg);

// argument check of sta_shared_forward (STA_OK or the failure code, message recorded)
int check_shared_forward(const sta_forward_args* a);

// global device error word (bounded waits that expired)
int* device_error_word();

int launch_rope_split(const void* x, int dtype, int64_t heads, int64_t N, int D,
                      int64_t stride_h, int64_t stride_n, const float* inv_freq,
                      float pos_scale, float rope_scale, void* hi, void* lo,
                      cudaStream_t stream, int mode = 0, int64_t dca_L = 0, int64_t dca_s = 0,
                      int64_t pos0 = 0, const void* tab = nullptr, float tab_R = 0.f,
                      int64_t tab_len = 0);

int launch_select(const sta_select_args* a, cudaStream_t stream);
size_t select_screen_bytes(const sta_select_args* a);
int launch_rope_table(const float* inv_freq, int D, float rope_scale, float R, int64_t len,
                      void* out, cudaStream_t stream);
int launch_build_sets(const sta_build_args* a, cudaStream_t stream);
int launch_build_sets_pq(const sta_build_pq_args* a, cudaStream_t stream);
int launch_build_sets_chunk(const sta_build_chunk_args* a, cudaStream_t stream);
int launch_gather_attend(const sta_attend_args* a, cudaStream_t stream);
int launch_pqstream(const sta_pqstream_args* a, cudaStream_t stream);
size_t decode_workspace_bytes(const sta_decode_args* a);
int decode_forward(const sta_decode_args* a, void* ws, size_t ws_len, cudaStream_t stream);

// cuTensorMapEncodeTiled obtained through the runtime's driver entry point
bool make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t d, uint64_t n,
                       uint64_t heads, uint32_t box_d, uint32_t box_rows);

}  // namespace sta
