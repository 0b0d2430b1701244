// stft_write_probe.cu — write ceiling of the stft output layout (a standalone
// program, not part of the library).
//
// The complex64 (C, F, S) = 64 x 1025 x 8189 output of the default stft
// workload has an odd row stride, so row runs start at every 8-byte phase of
// a 32-byte sector.  This program times writing the whole output with the
// patterns a store stage could use, from shared-memory staging rows, one CTA
// per SM.  Each CTA owns a contiguous run of 8-column tiles of one channel;
// for every tile and every bin row it writes the sector-aligned 64-byte run
// [col0 - phi_k, col0 - phi_k + 8) from a staging row (only runs entirely
// inside [0, S) are written).  Variants:
//   lsu_v2  NW warps of 8-byte stores (8 lanes per row, 4 rows an instruction)
//   lsu_v4  NW warps of 16-byte stores (4 lanes per row, 8 rows an instruction)
//   bulk    NW warps issuing one cp.async.bulk (a store-direction copy from
//           shared memory to this GPU's global memory) of 64 bytes per row
//           run; after each tile
//           the issuing threads wait until their copies have read shared
//           memory (wait_group.read LAG)
// and a cudaMemsetAsync of the whole output as the contiguous reference.
// Build and run (one B200):
//   nvcc -std=c++17 -gencode arch=compute_100a,code=sm_100a -O3 \
//        -o /tmp/stft_write_probe insight_b200/csrc/stft_write_probe.cu
//   /tmp/stft_write_probe
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include <vector>
#include <algorithm>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("ERR %s line %d: %s\n", #x, __LINE__, cudaGetErrorString(e)); return 1; } } while (0)

constexpr int C = 64, F = 1025, S = 8189;
constexpr int TW = 8;                       // columns per tile
constexpr int TPC = (S + TW - 1) / TW;      // tiles per channel (1024)
constexpr int ROWB = 144;                   // staging row stride in bytes
constexpr int SMEM = F * ROWB;              // 147600

struct Args { float2 *out; int nsub; };

__device__ __forceinline__ int phase_of(const float2 *p) {
  return (int)((reinterpret_cast<uintptr_t>(p) >> 3) & 3);
}

// V0: NW warps, st.global.v2 (8 B / lane: 8 lanes per row, 4 rows per instr)
template <int NW>
__global__ void __launch_bounds__(NW * 32) v_lsu_v2(Args a) {
  extern __shared__ __align__(16) unsigned char sm[];
  for (int i = threadIdx.x; i < SMEM / 4; i += blockDim.x) ((float *)sm)[i] = (float)i;
  __syncthreads();
  const int lane8 = threadIdx.x & 7, r0 = threadIdx.x >> 3;
  constexpr int RPI = NW * 32 / 8;
  const int upc = (TPC + a.nsub - 1) / a.nsub;
  for (int unit = blockIdx.x; unit < C * upc; unit += gridDim.x) {
    const int c = unit / upc, t0 = (unit - c * upc) * a.nsub;
    const int t1 = min(TPC, t0 + a.nsub);
    for (int t = t0; t < t1; ++t) {
      const int col0 = t * TW;
      for (int k = r0; k < F; k += RPI) {
        float2 *row = a.out + ((int64_t)c * F + k) * S;
        const int a0 = col0 - phase_of(row + col0);
        if (a0 >= 0 && a0 + 8 <= S) {
          float2 v = *(const float2 *)(sm + k * ROWB + lane8 * 8);
          row[a0 + lane8] = v;
        }
      }
      __syncthreads();
    }
  }
}

// V1: NW warps, st.global.v4 (16 B / lane: 4 lanes per row, 8 rows per instr)
template <int NW>
__global__ void __launch_bounds__(NW * 32) v_lsu_v4(Args a) {
  extern __shared__ __align__(16) unsigned char sm[];
  for (int i = threadIdx.x; i < SMEM / 4; i += blockDim.x) ((float *)sm)[i] = (float)i;
  __syncthreads();
  const int lane4 = threadIdx.x & 3, r0 = threadIdx.x >> 2;
  constexpr int RPI = NW * 32 / 4;
  const int upc = (TPC + a.nsub - 1) / a.nsub;
  for (int unit = blockIdx.x; unit < C * upc; unit += gridDim.x) {
    const int c = unit / upc, t0 = (unit - c * upc) * a.nsub;
    const int t1 = min(TPC, t0 + a.nsub);
    for (int t = t0; t < t1; ++t) {
      const int col0 = t * TW;
      for (int k = r0; k < F; k += RPI) {
        float2 *row = a.out + ((int64_t)c * F + k) * S;
        const int a0 = col0 - phase_of(row + col0);
        if (a0 >= 0 && a0 + 8 <= S) {
          float4 v = *(const float4 *)(sm + k * ROWB + lane4 * 16);
          *(float4 *)(row + a0 + 2 * lane4) = v;
        }
      }
      __syncthreads();
    }
  }
}

// V2: NW warps issue one cp.async.bulk (64 B, shared -> global) per row run;
// after each tile every issuing thread waits until its copies have read
// shared memory (wait_group.read LAG) before the next tile's barrier.
template <int NW, int LAG>
__global__ void __launch_bounds__(NW * 32) v_bulk(Args a) {
  extern __shared__ __align__(16) unsigned char sm[];
  for (int i = threadIdx.x; i < SMEM / 4; i += blockDim.x) ((float *)sm)[i] = (float)i;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(sm);
  const int upc = (TPC + a.nsub - 1) / a.nsub;
  for (int unit = blockIdx.x; unit < C * upc; unit += gridDim.x) {
    const int c = unit / upc, t0 = (unit - c * upc) * a.nsub;
    const int t1 = min(TPC, t0 + a.nsub);
    for (int t = t0; t < t1; ++t) {
      const int col0 = t * TW;
      for (int k = threadIdx.x; k < F; k += NW * 32) {
        float2 *row = a.out + ((int64_t)c * F + k) * S;
        const int a0 = col0 - phase_of(row + col0);
        if (a0 >= 0 && a0 + 8 <= S) {
          asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], 64;"
                       :: "l"(row + a0), "r"(sbase + k * ROWB) : "memory");
        }
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(LAG) : "memory");
      __syncthreads();
    }
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <typename K>
int run(const char *name, K kern, int threads, Args a, int sms, double bytes) {
  CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0)); CK(cudaEventCreate(&e1));
  kern<<<sms, threads, SMEM>>>(a);
  CK(cudaGetLastError()); CK(cudaDeviceSynchronize());
  std::vector<float> ms;
  for (int r = 0; r < 5; ++r) {
    CK(cudaEventRecord(e0));
    kern<<<sms, threads, SMEM>>>(a);
    CK(cudaEventRecord(e1));
    CK(cudaEventSynchronize(e1));
    float m; CK(cudaEventElapsedTime(&m, e0, e1)); ms.push_back(m);
  }
  std::sort(ms.begin(), ms.end());
  printf("%-16s best %.3f ms  median %.3f ms  %.2f TB/s (best)\n", name, ms[0], ms[2],
         bytes / (ms[0] * 1e-3) / 1e12);
  return 0;
}

int main() {
  int sms = 0; CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
  size_t n = (size_t)C * F * S;
  float2 *out; CK(cudaMalloc(&out, n * sizeof(float2)));
  CK(cudaMemset(out, 0, n * sizeof(float2)));
  Args a{out, 64};
  // written bytes: whole runs only (approximately all columns)
  double bytes = (double)n * 8;
  printf("SMs %d, nsub %d, output %.2f GB\n", sms, a.nsub, bytes / 1e9);
  if (run("lsu_v2 8w", v_lsu_v2<8>, 256, a, sms, bytes)) return 1;
  if (run("lsu_v2 16w", v_lsu_v2<16>, 512, a, sms, bytes)) return 1;
  if (run("lsu_v4 4w", v_lsu_v4<4>, 128, a, sms, bytes)) return 1;
  if (run("lsu_v4 8w", v_lsu_v4<8>, 256, a, sms, bytes)) return 1;
  if (run("bulk 1w lag0", v_bulk<1, 0>, 32, a, sms, bytes)) return 1;
  if (run("bulk 2w lag0", v_bulk<2, 0>, 64, a, sms, bytes)) return 1;
  if (run("bulk 4w lag0", v_bulk<4, 0>, 128, a, sms, bytes)) return 1;
  if (run("bulk 1w lag1", v_bulk<1, 1>, 32, a, sms, bytes)) return 1;
  if (run("bulk 4w lag1", v_bulk<4, 1>, 128, a, sms, bytes)) return 1;
  // contiguous reference: one big memset-like stream
  cudaEvent_t e0, e1; CK(cudaEventCreate(&e0)); CK(cudaEventCreate(&e1));
  CK(cudaEventRecord(e0)); CK(cudaMemsetAsync(out, 1, n * sizeof(float2))); CK(cudaEventRecord(e1));
  CK(cudaEventSynchronize(e1)); float m; CK(cudaEventElapsedTime(&m, e0, e1));
  printf("%-16s %.3f ms  %.2f TB/s\n", "memset", m, bytes / (m * 1e-3) / 1e12);
  CK(cudaFree(out));
  return 0;
}
