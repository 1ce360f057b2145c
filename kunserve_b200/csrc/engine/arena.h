// Parameter/KV memory arena on CUDA virtual memory management.
//
// Each decoder layer's weights live in their own physical allocation mapped
// into one contiguous weight range; the paged KV pool is a second range whose
// first part holds the base pages.  Dropping a layer (balloon) unmaps its
// physical memory from the weight range and maps it at the end of the KV
// range, where it becomes extend pages; restoring does the reverse.  This
// is the B200 counterpart of the reference's "parameter memory manager"
// (pmm_drop / pmm_restore, kunserve/worker.py:454-512).  Physical handles are
// created exportable as POSIX file descriptors so peer processes can map
// them for in-kernel P2P copies.
#pragma once
#include <cuda.h>

#include <cstdint>
#include <string>
#include <vector>

namespace kus {

struct DriverApi {
  CUresult (*memCreate)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long);
  CUresult (*memRelease)(CUmemGenericAllocationHandle);
  CUresult (*memAddressReserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  CUresult (*memAddressFree)(CUdeviceptr, size_t);
  CUresult (*memMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  CUresult (*memUnmap)(CUdeviceptr, size_t);
  CUresult (*memSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);
  CUresult (*memGetAllocationGranularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
  CUresult (*memExportToShareableHandle)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                                         unsigned long long);
  CUresult (*memImportFromShareableHandle)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  static const DriverApi& get();
};

void check_cu(CUresult r, const char* what);

struct Segment {
  CUmemGenericAllocationHandle handle = 0;
  size_t bytes = 0;         // physical size (granularity multiple)
  CUdeviceptr home = 0;     // address in the weight range
  CUdeviceptr mapped = 0;   // where it is mapped now (home, or inside the KV range)
};

class Arena {
 public:
  Arena(int device, const std::vector<size_t>& layer_bytes, size_t kv_base_bytes, bool exportable);
  ~Arena();
  Arena(const Arena&) = delete;
  Arena& operator=(const Arena&) = delete;

  char* layer_ptr(int l) const { return reinterpret_cast<char*>(segs_[l].home); }
  char* kv_base() const { return reinterpret_cast<char*>(kv_va_); }
  size_t kv_base_bytes() const { return kv_base_bytes_; }
  // whole reserved KV range: base pages plus room for every layer's extend pages
  size_t kv_va_bytes() const { return kv_va_bytes_; }
  // bytes mapped after the base pages: padding plus the dropped layers' memory
  size_t after_base_bytes() const { return ext_bytes_ + (kv_phys_bytes_ - kv_base_bytes_); }
  size_t granularity() const { return gran_; }
  size_t layer_bytes(int l) const { return segs_[l].bytes; }
  int num_layers() const { return (int)segs_.size(); }

  // Move the listed layers' memory behind the KV base pages; returns the
  // number of contiguous bytes now mapped after the base pages.
  size_t drop_layers(const std::vector<int>& layers);
  // Map dropped layers back at their weight address (contents are stale;
  // the caller refills them).  Returns the layers that were restored.
  std::vector<int> restore_layers();
  size_t extend_bytes() const { return ext_bytes_; }
  const std::vector<int>& dropped() const { return dropped_; }

  // POSIX fd of a layer's physical memory / of the KV base memory.
  int export_layer_fd(int l) const;
  int export_kv_fd() const;
  size_t kv_phys_bytes() const { return kv_phys_bytes_; }

 private:
  void map_rw(CUdeviceptr va, size_t bytes, CUmemGenericAllocationHandle h);
  int device_;
  size_t gran_ = 0;
  std::vector<Segment> segs_;
  CUdeviceptr w_va_ = 0;
  size_t w_va_bytes_ = 0;
  CUdeviceptr kv_va_ = 0;
  size_t kv_va_bytes_ = 0;
  size_t kv_base_bytes_ = 0;
  size_t kv_phys_bytes_ = 0;
  CUmemGenericAllocationHandle kv_handle_ = 0;
  size_t ext_bytes_ = 0;
  std::vector<int> dropped_;
  bool exportable_ = false;
};

// A standalone device buffer whose memory can be exported to peer processes
// (symmetric receive buffers of the fused TP kernels, P2P benchmarks).
class SharedBuffer {
 public:
  SharedBuffer(int device, size_t bytes);
  ~SharedBuffer();
  char* ptr() const { return reinterpret_cast<char*>(va_); }
  size_t bytes() const { return bytes_; }
  int export_fd() const;

 private:
  CUmemGenericAllocationHandle h_ = 0;
  CUdeviceptr va_ = 0;
  size_t bytes_ = 0;
};

// Map another process's exported physical memory (fd) into this context.
class PeerMapping {
 public:
  PeerMapping(int device, int fd, size_t bytes);
  ~PeerMapping();
  char* ptr() const { return reinterpret_cast<char*>(va_); }
  size_t bytes() const { return bytes_; }

 private:
  CUmemGenericAllocationHandle h_ = 0;
  CUdeviceptr va_ = 0;
  size_t bytes_ = 0;
};

}  // namespace kus
