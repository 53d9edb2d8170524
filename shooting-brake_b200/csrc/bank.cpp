// SBEXP001 expert-bank reader: the reference's on-disk NVFP4 bank (writer
// src/phase1/extract_experts.py:51-128, 234-281; C++ reader
// src/phase1/b70_provider.cpp:194-246, 866-934) mapped read-only and copied
// into the device layout of sbb200_nvfp4_moe.
//
// File: a packed 60-byte header {magic "SBEXP001", u32 layers, u32 experts
// per layer, u32 hidden, u32 intermediate, u32 reserved (0), u64 w13_bytes,
// u64 s13_bytes, u64 w2_bytes, u64 s2_bytes}, then one record per (layer,
// expert), layer-major: w13 [2I, H/2] (gate rows then up rows), s13
// [2I, H/16] e4m3, w2 [H, I/2], s2 [H, I/16], then two little-endian fp32
// dequant multipliers (w13's, w2's). The device layout is plane-major
// ([E, 2I, H/2] ...), so a layer load copies each expert's four planes to
// their rows of the four device planes; only the experts asked for (an
// expert-parallel shard) are read.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "kernels.h"
#include "sbb200.h"

namespace {

#pragma pack(push, 1)
struct BankHeader {
  char magic[8];
  uint32_t layers;
  uint32_t experts;
  uint32_t hidden;
  uint32_t intermediate;
  uint32_t reserved;
  uint64_t w13_bytes;
  uint64_t s13_bytes;
  uint64_t w2_bytes;
  uint64_t s2_bytes;
};
#pragma pack(pop)
static_assert(sizeof(BankHeader) == 60, "the packed bank header is 60 bytes");

int bank_fail(int code, const std::string& msg) {
  sbb::set_last_error(msg);
  return code;
}

}  // namespace

struct sbb200_bank {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t map_bytes = 0;
  BankHeader h{};
  uint64_t expert_bytes = 0;

  const uint8_t* record(size_t layer, size_t expert) const {
    return map + sizeof(BankHeader) + (layer * h.experts + expert) * expert_bytes;
  }
};

namespace {

void bank_release(sbb200_bank* b) {
  if (b->map) munmap(const_cast<uint8_t*>(b->map), b->map_bytes);
  if (b->fd >= 0) close(b->fd);
  delete b;
}

}  // namespace

extern "C" {

sbb200_bank_t* sbb200_bank_open(const char* path) {
  if (!path) {
    sbb::set_last_error("bank open: null path");
    return nullptr;
  }
  auto* b = new (std::nothrow) sbb200_bank();
  if (!b) return nullptr;
  auto reject = [&](const std::string& msg) -> sbb200_bank_t* {
    sbb::set_last_error(msg);
    bank_release(b);
    return nullptr;
  };
  b->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (b->fd < 0) return reject(std::string("open expert bank: ") + std::strerror(errno));
  struct stat st {};
  if (fstat(b->fd, &st) != 0) return reject(std::string("fstat expert bank: ") + std::strerror(errno));
  if (!S_ISREG(st.st_mode) || static_cast<uint64_t>(st.st_size) < sizeof(BankHeader))
    return reject("expert bank is not a regular file large enough to hold a header");
  b->map_bytes = static_cast<size_t>(st.st_size);
  void* m = mmap(nullptr, b->map_bytes, PROT_READ, MAP_SHARED, b->fd, 0);
  if (m == MAP_FAILED) {
    b->map_bytes = 0;
    return reject(std::string("mmap expert bank: ") + std::strerror(errno));
  }
  b->map = static_cast<const uint8_t*>(m);
  std::memcpy(&b->h, b->map, sizeof(BankHeader));
  if (std::memcmp(b->h.magic, "SBEXP001", 8) != 0) {
    std::string found(b->h.magic, b->h.magic + 8);
    for (char& c : found)
      if (c < 32 || c > 126) c = '?';
    return reject("expert bank magic '" + found + "' is unsupported; expected 'SBEXP001'");
  }
  const BankHeader& h = b->h;
  const uint64_t H = h.hidden, I = h.intermediate;
  if (h.reserved != 0)
    return reject("expert bank header does not match the NVFP4 bank contract (reserved != 0)");
  if (h.layers == 0 || h.experts == 0 || H == 0 || I == 0 || H % 16 || I % 16 ||
      h.w13_bytes != 2 * I * (H / 2) || h.s13_bytes != 2 * I * (H / 16) ||
      h.w2_bytes != H * (I / 2) || h.s2_bytes != H * (I / 16))
    return reject("expert bank header declares an inconsistent or unsupported geometry");
  b->expert_bytes = h.w13_bytes + h.s13_bytes + h.w2_bytes + h.s2_bytes + 2 * sizeof(float);
  const uint64_t expected =
      sizeof(BankHeader) + static_cast<uint64_t>(h.layers) * h.experts * b->expert_bytes;
  if (static_cast<uint64_t>(st.st_size) != expected)
    return reject("expert bank size does not match the geometry its header declares");
  return b;
}

int sbb200_bank_info(sbb200_bank_t* b, size_t* layers, size_t* experts, size_t* hidden,
                     size_t* intermediate) {
  if (!b) return bank_fail(SBB200_EINVAL, "bank info: null bank");
  if (layers) *layers = b->h.layers;
  if (experts) *experts = b->h.experts;
  if (hidden) *hidden = b->h.hidden;
  if (intermediate) *intermediate = b->h.intermediate;
  return SBB200_OK;
}

int sbb200_bank_read_expert(sbb200_bank_t* b, size_t layer, size_t expert, void* w13,
                            void* w13_scales, float* w13_global_scale, void* w2,
                            void* w2_scales, float* w2_global_scale) {
  if (!b) return bank_fail(SBB200_EINVAL, "bank read: null bank");
  if (layer >= b->h.layers || expert >= b->h.experts)
    return bank_fail(SBB200_EINVAL, "bank read: layer or expert outside the bank");
  const uint8_t* r = b->record(layer, expert);
  const BankHeader& h = b->h;
  if (w13) std::memcpy(w13, r, h.w13_bytes);
  r += h.w13_bytes;
  if (w13_scales) std::memcpy(w13_scales, r, h.s13_bytes);
  r += h.s13_bytes;
  if (w2) std::memcpy(w2, r, h.w2_bytes);
  r += h.w2_bytes;
  if (w2_scales) std::memcpy(w2_scales, r, h.s2_bytes);
  r += h.s2_bytes;
  if (w13_global_scale) std::memcpy(w13_global_scale, r, sizeof(float));
  if (w2_global_scale) std::memcpy(w2_global_scale, r + sizeof(float), sizeof(float));
  return SBB200_OK;
}

int sbb200_bank_load(sbb200_bank_t* b, void* stream, size_t layer, size_t expert_begin,
                     size_t expert_count, void* w13, void* w13_scales,
                     float* w13_global_scales, void* w2, void* w2_scales,
                     float* w2_global_scales) {
  if (!b) return bank_fail(SBB200_EINVAL, "bank load: null bank");
  if (layer >= b->h.layers || expert_begin > b->h.experts ||
      expert_count > b->h.experts - expert_begin)
    return bank_fail(SBB200_EINVAL, "bank load: layer or expert range outside the bank");
  if (!w13 || !w13_scales || !w13_global_scales || !w2 || !w2_scales || !w2_global_scales)
    return bank_fail(SBB200_EINVAL, "bank load: null device pointer");
  const BankHeader& h = b->h;
  auto s = static_cast<cudaStream_t>(stream);
  // pinned staging for one record at a time, double-buffered so the copy of
  // one expert overlaps the host read of the next
  uint8_t* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
    e = cudaMallocHost(reinterpret_cast<void**>(&stage[i]), b->expert_bytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
  }
  std::vector<float> g13(expert_count), g2(expert_count);
  for (size_t i = 0; i < expert_count && e == cudaSuccess; ++i) {
    const int k = static_cast<int>(i & 1);
    e = cudaEventSynchronize(done[k]);  // the buffer's previous copies are done
    if (e != cudaSuccess) break;
    std::memcpy(stage[k], b->record(layer, expert_begin + i), b->expert_bytes);
    const uint8_t* r = stage[k];
    e = cudaMemcpyAsync(static_cast<uint8_t*>(w13) + i * h.w13_bytes, r, h.w13_bytes,
                        cudaMemcpyHostToDevice, s);
    r += h.w13_bytes;
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<uint8_t*>(w13_scales) + i * h.s13_bytes, r, h.s13_bytes,
                          cudaMemcpyHostToDevice, s);
    r += h.s13_bytes;
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<uint8_t*>(w2) + i * h.w2_bytes, r, h.w2_bytes,
                          cudaMemcpyHostToDevice, s);
    r += h.w2_bytes;
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<uint8_t*>(w2_scales) + i * h.s2_bytes, r, h.s2_bytes,
                          cudaMemcpyHostToDevice, s);
    r += h.s2_bytes;
    std::memcpy(&g13[i], r, sizeof(float));
    std::memcpy(&g2[i], r + sizeof(float), sizeof(float));
    if (e == cudaSuccess) e = cudaEventRecord(done[k], s);
  }
  if (e == cudaSuccess && expert_count)
    e = cudaMemcpyAsync(w13_global_scales, g13.data(), expert_count * sizeof(float),
                        cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && expert_count)
    e = cudaMemcpyAsync(w2_global_scales, g2.data(), expert_count * sizeof(float),
                        cudaMemcpyHostToDevice, s);
  // the staging buffers and g13/g2 are released below: finish every copy
  const cudaError_t se = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = se;
  for (int i = 0; i < 2; ++i) {
    if (done[i]) cudaEventDestroy(done[i]);
    if (stage[i]) cudaFreeHost(stage[i]);
  }
  if (e != cudaSuccess)
    return bank_fail(SBB200_ECUDA, std::string("bank load: ") + cudaGetErrorString(e));
  return SBB200_OK;
}

void sbb200_bank_close(sbb200_bank_t* b) {
  if (b) bank_release(b);
}

}  // extern "C"
