// Host program: float32 values (file) -> e4m3 bytes with CUDA's own conversion
// (__nv_cvt_float_to_fp8, round-to-nearest-even, saturating), used by tests/test_fp8_cpu.py to
// pin the oracle's e4m3 rounding. Host code only; built with nvcc, no GPU needed.
#include <cuda_fp8.h>
#include <cstdio>
#include <vector>

int main(int argc, char** argv) {
  if (argc != 3) return 2;
  FILE* f = fopen(argv[1], "rb");
  if (!f) return 3;
  std::vector<float> x;
  float buf[4096];
  size_t n;
  while ((n = fread(buf, sizeof(float), 4096, f)) > 0) x.insert(x.end(), buf, buf + n);
  fclose(f);
  std::vector<unsigned char> o(x.size());
  for (size_t i = 0; i < x.size(); ++i)
    o[i] = __nv_cvt_float_to_fp8(x[i], __NV_SATFINITE, __NV_E4M3);
  FILE* g = fopen(argv[2], "wb");
  if (!g) return 4;
  fwrite(o.data(), 1, o.size(), g);
  fclose(g);
  return 0;
}
