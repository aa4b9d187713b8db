/* The C ABI used from plain C (no C++): the header compiles as C99, every host-side
 * entry that needs no GPU answers as documented.  Built and run by tests/test_c_abi.py. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "w4a16_b200.h"

static int failures = 0;

static void expect(int cond, const char* what) {
  if (!cond) {
    fprintf(stderr, "FAIL: %s\n", what);
    ++failures;
  }
}

int main(void) {
  const uint8_t* packed = (const uint8_t*)(uintptr_t)4096;
  const void* scale = (const void*)(uintptr_t)4096;
  const void* x = (const void*)(uintptr_t)65536;
  void* out = (void*)(uintptr_t)8192;

  expect(w4a16_version() == 10000, "version");
  expect(strcmp(w4a16_status_string(W4A16_OK), "ok") == 0, "status string ok");
  expect(w4a16_status_string(W4A16_ERR_SHAPE) != NULL, "status string shape");

  /* validation happens before any CUDA call */
  expect(w4a16_gemv(packed, W4A16_PACK_INTERLEAVED, scale, W4A16_DTYPE_F32, 64, x, 1, 16, 256, out,
                    W4A16_DTYPE_F32, NULL, NULL, 0, NULL) == W4A16_ERR_DTYPE, "group 64 rejected");
  expect(w4a16_gemv(packed, W4A16_PACK_INTERLEAVED, scale, W4A16_DTYPE_F32, 0, x, 1, 16, 12, out,
                    W4A16_DTYPE_F32, NULL, NULL, 0, NULL) == W4A16_ERR_SHAPE, "cols 12 rejected");
  expect(strstr(w4a16_last_error_string(), "12") != NULL, "last error names the bad value");
  expect(w4a16_gemv(NULL, W4A16_PACK_INTERLEAVED, scale, W4A16_DTYPE_F32, 0, x, 1, 16, 256, out,
                    W4A16_DTYPE_F32, NULL, NULL, 0, NULL) == W4A16_ERR_NULL, "null packed rejected");
  expect(w4a16_gemv(packed, W4A16_PACK_INTERLEAVED, scale, W4A16_DTYPE_F32, 0, x, 1, 0, 256, out,
                    W4A16_DTYPE_F32, NULL, NULL, 0, NULL) == W4A16_OK, "empty problem is a no-op");
  expect(w4a16_marlin_g128_cuda(NULL, NULL, NULL, NULL, 16, 256, NULL) == W4A16_ERR_NULL,
         "reference-named entry validates");
  expect(w4a16_gemv_fused(packed, scale, W4A16_DTYPE_F32, 128, 9, x, NULL, 1e-5f, 16, 256, out,
                          W4A16_DTYPE_F32, NULL, NULL, 0, 0u, NULL) == W4A16_ERR_DTYPE,
         "unknown prologue rejected");
  expect(w4a16_gemv_workspace_bytes(1, 262144, 2048) > 0, "workspace size");
  expect(w4a16_decode_attention_scratch_bytes(32, 8, 16) == (size_t)(32 * 16 * 66 + 8) * 4,
         "attention scratch size");
  expect(w4a16_tp_header_bytes() == 256 && w4a16_tp_ipc_handle_bytes() == 64, "tp sizes");
  {
    void* regions[2] = {(void*)(uintptr_t)(1 << 20), (void*)(uintptr_t)(2 << 20)};
    expect(w4a16_gemv_allgather(packed, scale, W4A16_DTYPE_F32, 0, x, 16, 256, W4A16_DTYPE_F32, 0, 2, 2,
                                regions, NULL, 0, 0u, NULL) == W4A16_ERR_SHAPE,
           "allgather rank out of range rejected");
    /* regions this process neither allocated nor opened are rejected before any launch */
    expect(w4a16_gemv_allgather(packed, scale, W4A16_DTYPE_F32, 0, x, 16, 256, W4A16_DTYPE_F32, 0, 0, 2,
                                regions, NULL, 0, 0u, NULL) == W4A16_ERR_SHAPE,
           "allgather into unknown regions rejected");
    expect(strstr(w4a16_last_error_string(), "w4a16_tp_region_alloc") != NULL,
           "unknown region error names the allocator");
  }
  expect(w4a16_tp_set_peer_wait_ns(1ull) == W4A16_ERR_SHAPE, "1 ns peer wait rejected");
  expect(w4a16_tp_set_peer_wait_ns(100000000ull) == W4A16_OK, "100 ms peer wait accepted");
  expect(w4a16_tp_set_peer_wait_ns(0ull) == W4A16_OK, "peer wait default restored");
  if (failures == 0) printf("c abi ok\n");
  return failures == 0 ? 0 : 1;
}
