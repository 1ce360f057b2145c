#include "arena.h"

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace kus {

void check_cu(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) throw std::runtime_error(std::string("CUDA driver call failed: ") + what + " (" +
                                                  std::to_string((int)r) + ")");
}

template <typename F>
static void load(F& fn, const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || !p)
    throw std::runtime_error(std::string("driver entry point missing: ") + name);
  fn = reinterpret_cast<F>(p);
}

const DriverApi& DriverApi::get() {
  static DriverApi api = [] {
    DriverApi a{};
    load(a.memCreate, "cuMemCreate");
    load(a.memRelease, "cuMemRelease");
    load(a.memAddressReserve, "cuMemAddressReserve");
    load(a.memAddressFree, "cuMemAddressFree");
    load(a.memMap, "cuMemMap");
    load(a.memUnmap, "cuMemUnmap");
    load(a.memSetAccess, "cuMemSetAccess");
    load(a.memGetAllocationGranularity, "cuMemGetAllocationGranularity");
    load(a.memExportToShareableHandle, "cuMemExportToShareableHandle");
    load(a.memImportFromShareableHandle, "cuMemImportFromShareableHandle");
    return a;
  }();
  return api;
}

static CUmemAllocationProp make_prop(int device, bool exportable) {
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = exportable ? CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR : CU_MEM_HANDLE_TYPE_NONE;
  return p;
}

static size_t round_up(size_t x, size_t g) { return (x + g - 1) / g * g; }

void Arena::map_rw(CUdeviceptr va, size_t bytes, CUmemGenericAllocationHandle h) {
  const auto& d = DriverApi::get();
  check_cu(d.memMap(va, bytes, 0, h, 0), "cuMemMap");
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device_;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  check_cu(d.memSetAccess(va, bytes, &acc, 1), "cuMemSetAccess");
}

Arena::Arena(int device, const std::vector<size_t>& layer_bytes, size_t kv_base_bytes, bool exportable)
    : device_(device), exportable_(exportable) {
  const auto& d = DriverApi::get();
  CUmemAllocationProp prop = make_prop(device, exportable);
  check_cu(d.memGetAllocationGranularity(&gran_, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "granularity");
  size_t total_w = 0;
  for (size_t b : layer_bytes) total_w += round_up(b ? b : 1, gran_);
  w_va_bytes_ = total_w ? total_w : gran_;
  check_cu(d.memAddressReserve(&w_va_, w_va_bytes_, gran_, 0, 0), "reserve weights");
  CUdeviceptr cur = w_va_;
  for (size_t b : layer_bytes) {
    Segment s;
    s.bytes = round_up(b ? b : 1, gran_);
    check_cu(d.memCreate(&s.handle, s.bytes, &prop, 0), "cuMemCreate layer");
    s.home = cur;
    s.mapped = cur;
    map_rw(cur, s.bytes, s.handle);
    cur += s.bytes;
    segs_.push_back(s);
  }
  kv_base_bytes_ = kv_base_bytes;
  kv_phys_bytes_ = round_up(kv_base_bytes ? kv_base_bytes : 1, gran_);
  kv_va_bytes_ = kv_phys_bytes_ + total_w + gran_;
  check_cu(d.memAddressReserve(&kv_va_, kv_va_bytes_, gran_, 0, 0), "reserve kv");
  check_cu(d.memCreate(&kv_handle_, kv_phys_bytes_, &prop, 0), "cuMemCreate kv");
  map_rw(kv_va_, kv_phys_bytes_, kv_handle_);
}

Arena::~Arena() {
  const auto& d = DriverApi::get();
  cudaDeviceSynchronize();
  for (auto& s : segs_) {
    if (s.mapped) d.memUnmap(s.mapped, s.bytes);
    d.memRelease(s.handle);
  }
  if (kv_handle_) {
    d.memUnmap(kv_va_, kv_phys_bytes_);
    d.memRelease(kv_handle_);
  }
  if (kv_va_) d.memAddressFree(kv_va_, kv_va_bytes_);
  if (w_va_) d.memAddressFree(w_va_, w_va_bytes_);
}

size_t Arena::drop_layers(const std::vector<int>& layers) {
  const auto& d = DriverApi::get();
  cudaDeviceSynchronize();
  for (int l : layers) {
    Segment& s = segs_.at(l);
    if (s.mapped != s.home) continue;   // already dropped
    check_cu(d.memUnmap(s.home, s.bytes), "unmap layer");
    const CUdeviceptr dst = kv_va_ + kv_phys_bytes_ + ext_bytes_;
    map_rw(dst, s.bytes, s.handle);
    s.mapped = dst;
    ext_bytes_ += s.bytes;
    dropped_.push_back(l);
  }
  // the extend region starts right after the (possibly padded) base pages
  return ext_bytes_ + (kv_phys_bytes_ - kv_base_bytes_);
}

std::vector<int> Arena::restore_layers() {
  const auto& d = DriverApi::get();
  cudaDeviceSynchronize();
  std::vector<int> out = dropped_;
  for (int l : dropped_) {
    Segment& s = segs_.at(l);
    check_cu(d.memUnmap(s.mapped, s.bytes), "unmap extend");
    map_rw(s.home, s.bytes, s.handle);
    s.mapped = s.home;
  }
  dropped_.clear();
  ext_bytes_ = 0;
  return out;
}

int Arena::export_layer_fd(int l) const {
  int fd = -1;
  check_cu(DriverApi::get().memExportToShareableHandle(&fd, segs_.at(l).handle,
                                                       CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
           "export layer");
  return fd;
}

int Arena::export_kv_fd() const {
  int fd = -1;
  check_cu(DriverApi::get().memExportToShareableHandle(&fd, kv_handle_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
           "export kv");
  return fd;
}

SharedBuffer::SharedBuffer(int device, size_t bytes) {
  const auto& d = DriverApi::get();
  CUmemAllocationProp prop = make_prop(device, true);
  size_t gran = 0;
  check_cu(d.memGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "granularity");
  bytes_ = round_up(bytes ? bytes : 1, gran);
  check_cu(d.memCreate(&h_, bytes_, &prop, 0), "cuMemCreate shared");
  check_cu(d.memAddressReserve(&va_, bytes_, gran, 0, 0), "reserve shared");
  check_cu(d.memMap(va_, bytes_, 0, h_, 0), "map shared");
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  check_cu(d.memSetAccess(va_, bytes_, &acc, 1), "access shared");
}

SharedBuffer::~SharedBuffer() {
  const auto& d = DriverApi::get();
  cudaDeviceSynchronize();
  if (va_) {
    d.memUnmap(va_, bytes_);
    d.memAddressFree(va_, bytes_);
  }
  if (h_) d.memRelease(h_);
}

int SharedBuffer::export_fd() const {
  int fd = -1;
  check_cu(DriverApi::get().memExportToShareableHandle(&fd, h_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
           "export shared");
  return fd;
}

PeerMapping::PeerMapping(int device, int fd, size_t bytes) : bytes_(bytes) {
  const auto& d = DriverApi::get();
  check_cu(d.memImportFromShareableHandle(&h_, reinterpret_cast<void*>((uintptr_t)fd),
                                          CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
           "import handle");
  CUmemAllocationProp prop = make_prop(device, true);
  size_t gran = 0;
  check_cu(d.memGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "granularity");
  check_cu(d.memAddressReserve(&va_, bytes_, gran, 0, 0), "reserve peer");
  check_cu(d.memMap(va_, bytes_, 0, h_, 0), "map peer");
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  check_cu(d.memSetAccess(va_, bytes_, &acc, 1), "access peer");
}

PeerMapping::~PeerMapping() {
  const auto& d = DriverApi::get();
  if (va_) {
    d.memUnmap(va_, bytes_);
    d.memAddressFree(va_, bytes_);
  }
  if (h_) d.memRelease(h_);
}

}  // namespace kus
