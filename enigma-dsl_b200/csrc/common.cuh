// common.cuh — shared declarations of the libenigma_cuda translation units.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "../../include/enigma_cuda.h"
#include "sm100.cuh"

namespace enigma {

// SM count of the current device (cached per device).
int sm_count();

// Device word that bounded waits set on timeout (one per device, zeroed at init; created
// by the first call, nullptr if that allocation fails).
uint32_t* device_status();
// The same word if it already exists on the current device, else nullptr (never allocates).
uint32_t* device_status_if_exists();
// A pair of work counters of the current device for one launch (a dynamic work queue:
// [0] next item, [1] spare), taken round-robin from a per-device pool so launches in flight
// on different streams use different pairs; the caller zeroes it on its stream before the
// launch.  nullptr if the per-device state could not be created.
uint32_t* work_counters();
// Reads and clears the no-allocation decode entry's status word on the current device
// (0 if that entry has not run there).  Allocates nothing.
cudaError_t noalloc_take_status(uint32_t* value);
// One CTA that waits on a barrier nothing arrives on, gives up after `polls` polls and
// flags *status as a timed-out bounded wait does.
cudaError_t launch_timeout_probe(uint32_t* status, long long polls, cudaStream_t s);

// Operator launchers (asynchronous).  Arguments are validated by the C ABI layer.
cudaStream_t aux_stream();
cudaError_t rmsnorm_launch(int dtype, const void* x, const void* w, void* y, int64_t rows,
                           int64_t hidden, float eps, cudaStream_t s);
// Same, with the SM count given (no per-device state is touched).
cudaError_t rmsnorm_launch_sms(int dtype, const void* x, const void* w, void* y, int64_t rows,
                               int64_t hidden, float eps, int sms, cudaStream_t s);
// The decode step's input norm (bf16): launched as a programmatic dependent when the row
// is at most 128 16-byte vectors (hidden <= 1024), so in a layer stack it is resident
// before the previous layer's last kernel ends; else the same as rmsnorm_launch_sms.
cudaError_t rmsnorm_launch_pdl_bf16(const void* x, const void* w, void* y, int64_t rows,
                                    int64_t hidden, float eps, int sms, cudaStream_t s);
cudaError_t gemm_bf16_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                             int64_t K, cudaStream_t s);
cudaError_t gemm_f32_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                            int64_t K, bool accumulate, cudaStream_t s);
cudaError_t gemm_f32_trans_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                  int64_t K, bool trans_a, bool trans_b, bool accumulate,
                                  cudaStream_t s);
cudaError_t sdpa_f32_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                            int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                            float scale, bool causal, cudaStream_t s);
cudaError_t sdpa_strided_launch(int dtype, const void* Q, const void* K, const void* V, void* O,
                                int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv,
                                int64_t D, const int64_t* strides12, float scale, bool causal,
                                const float* sinks, cudaStream_t s);
cudaError_t sdpa_bf16_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                             int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                             float scale, bool causal, cudaStream_t s);

size_t decode_workspace_bytes(const enigma_decode_layer_desc& d);
cudaError_t decode_layer_launch(const enigma_decode_layer_desc& d, const void* x, void* out,
                                void* ws, cudaStream_t s);

// Argument checks of a decode-layer descriptor (ENIGMA_OK or ENIGMA_ERR_BADARG + message).
int32_t check_decode_desc(const enigma_decode_layer_desc* d);

cudaError_t qwen_decode_f32_launch(const enigma_qwen_decode_f32_desc& q, cudaStream_t s);

cudaError_t elementwise_launch(int op, int dtype, const void* a, const void* b, void* c, int64_t n,
                               cudaStream_t s);

// Records the name of the device kernel an operator launcher chose, for
// enigma_last_kernel on the calling thread (a static string).
void note_kernel(const char* name);

// Records a message for enigma_last_error on the calling thread.
void set_error(const char* fmt, ...);

}  // namespace enigma
