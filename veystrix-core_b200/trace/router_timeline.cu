// Timeline of one fused router launch (router_fused_kernel, vx_router.cu):
// the library source is compiled with VX_STAMP recording %globaltimer per CTA
// at its numbered trace points, and the phases of the last CTA of every token
// block (top-k) and of the final CTA (the permutation) are printed relative to
// the first CTA's start.  Synthetic bf16 router weights and tokens at the
// benchmark shape (E = 512, d = 2048, k = 10); T from the command line.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -I include \
//        -I veystrix-core_b200/csrc veystrix-core_b200/trace/router_timeline.cu -o router_timeline
//   ./router_timeline 64
//
// Slots: 0 CTA start, 1 logits tile done, 2 last CTA of a token block starts
// the top-k, 9 its logits loads issued, 10 softmax done, 11 selection rounds
// done, 3 top-k done, 4 the final CTA starts the permutation, 5 ids counted,
// 6 run offsets, 7 positions ranked, 8 permutation done.
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <cuda_runtime.h>
__device__ unsigned long long g_stamp[512][12];
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define VX_STAMP(slot) \
  do { if (threadIdx.x == 0) g_stamp[blockIdx.y * gridDim.x + blockIdx.x][slot] = gtimer(); } while (0)
#include "../csrc/vx_router.cu"
namespace vx {
bool chain_enabled(bool) { return false; }
int sm_count() { return 148; }
}  // namespace vx

int main(int argc, char** argv) {
  using namespace vx;
  const int T = argc > 1 ? atoi(argv[1]) : 1, E = 512, K = 2048, k = 10;
  const int nTB = (T + 7) / 8, nEB = E / 16;
  std::vector<uint16_t> hx(size_t(T) * K), hw(size_t(E) * K), hs(K / 32), hb(K / 32);
  std::vector<uint32_t> hq(K / 8);
  unsigned s = 1;
  auto rnd = [&]() { s = s * 1664525u + 1013904223u; return s; };
  for (auto& v : hx) v = uint16_t(((rnd() >> 31) << 15) | (0x3E00 + (rnd() >> 24) % 200));
  for (auto& v : hw) v = uint16_t(((rnd() >> 31) << 15) | (0x3800 + (rnd() >> 24) % 300));
  for (auto& v : hq) v = rnd();
  for (auto& v : hs) v = 0x3A00;
  for (auto& v : hb) v = 0xBB00;
  uint16_t *x, *w, *lg, *wt, *sg, *sc, *bi;
  uint32_t* q;
  int32_t *inds, *cnt, *ord, *inv, *off, *act, *nact, *srow, *err, *items, *nit;
  const int P = T * k;
  cudaMalloc(&x, hx.size() * 2);
  cudaMalloc(&w, hw.size() * 2);
  cudaMalloc(&lg, size_t(T) * E * 2);
  cudaMalloc(&wt, P * 2);
  cudaMalloc(&sg, T * 2);
  cudaMalloc(&sc, hs.size() * 2);
  cudaMalloc(&bi, hb.size() * 2);
  cudaMalloc(&q, hq.size() * 4);
  cudaMalloc(&inds, P * 4);
  cudaMalloc(&cnt, (nTB + 1) * 4);
  cudaMalloc(&ord, P * 4);
  cudaMalloc(&inv, P * 4);
  cudaMalloc(&off, (E + 2) * 4);
  cudaMalloc(&act, (E + 1) * 4);
  cudaMalloc(&nact, 4);
  cudaMalloc(&srow, (P + T) * 4);
  cudaMalloc(&err, 8);
  cudaMalloc(&items, 3 * (P + T + E) * 4);
  cudaMalloc(&nit, 4);
  cudaMemset(err, 0, 8);
  cudaMemcpy(x, hx.data(), hx.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(w, hw.data(), hw.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(q, hq.data(), hq.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(sc, hs.data(), hs.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(bi, hb.data(), hb.size() * 2, cudaMemcpyHostToDevice);
  vx_q4 seg{};
  seg.w = q;
  seg.scales = sc;
  seg.biases = bi;
  seg.experts = 1;
  seg.out = 1;
  seg.in = K;
  seg.group_size = 32;
  PermSmallArgs pa{E, T, k, 4, nullptr, ord, inv, off, act, nact, srow, err, items, nit};
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  static unsigned long long z[512][12], st[512][12];
  for (int it = 0; it < 40; ++it) {
    cudaMemcpyToSymbol(g_stamp, z, sizeof(z));
    cudaEventRecord(e0);
    cudaError_t e = launch_router_fused(x, T, w, E, K, k, &seg, lg, inds, wt, sg, cnt, &pa, nullptr, 0);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    if (e != cudaSuccess) { printf("launch error %s\n", cudaGetErrorString(e)); return 1; }
    if (it < 37) continue;
    float ms;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaMemcpyFromSymbol(st, g_stamp, sizeof(st));
    const int gx = nEB + 1;
    unsigned long long t0 = ~0ull, smax = 0, mmax = 0;
    for (int b = 0; b < gx * nTB; ++b)
      if (st[b][0] && st[b][0] < t0) t0 = st[b][0];
    for (int b = 0; b < gx * nTB; ++b) {
      if (b % gx == nEB) continue;
      if (st[b][0] - t0 > smax) smax = st[b][0] - t0;
      if (st[b][1] - t0 > mmax) mmax = st[b][1] - t0;
    }
    printf("T=%d iter %d: event %.2f us; CTA start spread %.2f; MMA done max %.2f us\n", T, it, ms * 1e3,
           smax / 1e3, mmax / 1e3);
    for (int b = 0; b < gx * nTB; ++b) {
      if (st[b][2]) printf("  tb %d last CTA %d: top-k from %.2f, loaded %.2f, softmax %.2f, rounds %.2f, done %.2f", b / gx, b % gx,
                           (st[b][2] - t0) / 1e3, (st[b][9] - t0) / 1e3, (st[b][10] - t0) / 1e3, (st[b][11] - t0) / 1e3, (st[b][3] - t0) / 1e3);
      if (st[b][4]) printf(" | perm from %.2f, counted %.2f, offsets %.2f, ranked %.2f, end %.2f",
                           (st[b][4] - t0) / 1e3, (st[b][5] - t0) / 1e3, (st[b][6] - t0) / 1e3,
                           (st[b][7] - t0) / 1e3, (st[b][8] - t0) / 1e3);
      if (st[b][2]) printf("\n");
    }
  }
  int herr[2], hn[2];
  cudaMemcpy(herr, err, 8, cudaMemcpyDeviceToHost);
  cudaMemcpy(&hn[0], nact, 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(&hn[1], nit, 4, cudaMemcpyDeviceToHost);
  printf("err %d, n_active %d, n_items %d, status %s\n", herr[0], hn[0], hn[1],
         cudaGetErrorString(cudaDeviceSynchronize()));
  return 0;
}
