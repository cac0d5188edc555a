// Virtual-memory regions whose physical backing can be released and restored at the same address.
//
// The reference's inference engine hands the card to a colocated trainer by
// releasing its KV cache and weights (SGLang + torch_memory_saver,
// ``/release_memory_occupation`` / ``/resume_memory_occupation``) while keeping
// their virtual addresses, so CUDA graphs captured over them stay valid.  This
// is the same mechanism on the CUDA driver's virtual memory API: a region
// reserves a VA range once (cuMemAddressReserve); ``map`` creates physical
// memory (cuMemCreate), maps it into the range and enables access; ``unmap``
// unmaps and releases the physical memory, keeping the range.  Contents do not
// survive an unmap (callers that need them copy to host first).
//
// Driver entry points are resolved at run time through the runtime's
// cudaGetDriverEntryPoint, so the library does not link libcuda directly.
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "include/common.cuh"

namespace meshy {
namespace {

template <typename F>
F entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  MESHY_CUDA_CHECK(cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q));
  MESHY_CHECK(q == cudaDriverEntryPointSuccess && p, std::string("driver entry point missing: ") + name);
  return reinterpret_cast<F>(p);
}

struct Driver {
  decltype(&cuMemCreate) create;
  decltype(&cuMemRelease) release;
  decltype(&cuMemAddressReserve) reserve;
  decltype(&cuMemAddressFree) addr_free;
  decltype(&cuMemMap) map;
  decltype(&cuMemUnmap) unmap;
  decltype(&cuMemSetAccess) set_access;
  decltype(&cuMemGetAllocationGranularity) granularity;
};

const Driver& drv() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    d.create = entry<decltype(&cuMemCreate)>("cuMemCreate");
    d.release = entry<decltype(&cuMemRelease)>("cuMemRelease");
    d.reserve = entry<decltype(&cuMemAddressReserve)>("cuMemAddressReserve");
    d.addr_free = entry<decltype(&cuMemAddressFree)>("cuMemAddressFree");
    d.map = entry<decltype(&cuMemMap)>("cuMemMap");
    d.unmap = entry<decltype(&cuMemUnmap)>("cuMemUnmap");
    d.set_access = entry<decltype(&cuMemSetAccess)>("cuMemSetAccess");
    d.granularity = entry<decltype(&cuMemGetAllocationGranularity)>("cuMemGetAllocationGranularity");
  });
  return d;
}

void check(CUresult r, const char* what) {
  MESHY_CHECK(r == CUDA_SUCCESS, std::string(what) + " failed (CUresult " + std::to_string((int)r) + ")");
}

class VmmRegion {
 public:
  VmmRegion(int64_t nbytes, int device) : device_(device) {
    MESHY_CHECK(nbytes > 0, "VmmRegion: size must be positive");
    prop_ = {};
    prop_.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop_.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop_.location.id = device;
    size_t gran = 0;
    check(drv().granularity(&gran, &prop_, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "cuMemGetAllocationGranularity");
    size_ = ((size_t)nbytes + gran - 1) / gran * gran;
    check(drv().reserve(&va_, size_, gran, 0, 0), "cuMemAddressReserve");
    map();
  }
  ~VmmRegion() {
    try {
      if (mapped_) unmap();
      if (va_) drv().addr_free(va_, size_);
    } catch (...) {
    }
  }
  void map() {
    if (mapped_) return;
    check(drv().create(&handle_, size_, &prop_, 0), "cuMemCreate");
    check(drv().map(va_, size_, 0, handle_, 0), "cuMemMap");
    CUmemAccessDesc acc = {};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = device_;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    check(drv().set_access(va_, size_, &acc, 1), "cuMemSetAccess");
    mapped_ = true;
  }
  void unmap() {
    if (!mapped_) return;
    MESHY_CUDA_CHECK(cudaDeviceSynchronize());  // nothing may still be using the pages
    check(drv().unmap(va_, size_), "cuMemUnmap");
    check(drv().release(handle_), "cuMemRelease");
    mapped_ = false;
  }
  int64_t ptr() const { return (int64_t)va_; }
  int64_t size() const { return (int64_t)size_; }
  bool mapped() const { return mapped_; }
  // Non-owning tensor over [offset, offset + numel * itemsize): valid while the region is mapped, and
  // at the same address after a later map.
  torch::Tensor view(int64_t offset, std::vector<int64_t> shape, c10::ScalarType dtype) {
    int64_t numel = 1;
    for (auto s : shape) numel *= s;
    MESHY_CHECK(offset >= 0 && offset + numel * (int64_t)c10::elementSize(dtype) <= (int64_t)size_,
                "VmmRegion.view out of range");
    auto opts = torch::TensorOptions().device(torch::kCUDA, device_).dtype(dtype);
    return torch::from_blob(reinterpret_cast<char*>(va_) + offset, shape, opts);
  }

 private:
  int device_;
  CUmemAllocationProp prop_;
  CUdeviceptr va_ = 0;
  size_t size_ = 0;
  CUmemGenericAllocationHandle handle_ = 0;
  bool mapped_ = false;
};

}  // namespace

void register_vmm(pybind11::module_& m) {
  pybind11::class_<VmmRegion>(m, "VmmRegion",
                              "device memory with a stable virtual address whose physical pages can be released")
      .def(pybind11::init<int64_t, int>(), pybind11::arg("nbytes"), pybind11::arg("device"))
      .def("map", &VmmRegion::map, "create and map physical memory (contents undefined)")
      .def("unmap", &VmmRegion::unmap, "release the physical memory; the address range stays reserved")
      .def_property_readonly("ptr", &VmmRegion::ptr)
      .def_property_readonly("size", &VmmRegion::size)
      .def_property_readonly("mapped", &VmmRegion::mapped)
      .def("view", &VmmRegion::view, pybind11::arg("offset"), pybind11::arg("shape"), pybind11::arg("dtype"));
}

}  // namespace meshy
