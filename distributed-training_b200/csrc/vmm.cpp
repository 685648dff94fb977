// Peer memory through the CUDA virtual-memory-management API, shared by file descriptor.
//
// The default peer memory of NVLinkGroup is cudaMalloc + cudaIpc handles: an IPC
// mapping is tied to the exporting process's allocation, so a rank that dies takes
// the memory its peers are reading with it.  Here each rank creates a physical
// allocation with cuMemCreate (shareable as a POSIX file descriptor), maps it into its
// own address space, and passes the descriptor to its peers (over a Unix socket, in
// Python); a peer imports the descriptor, which holds its own reference to the
// physical memory, and maps it too.  The memory stays valid in every process that
// mapped it until that process unmaps it, whatever happens to the exporter.
//
// Driver entry points are resolved at run time through cudaGetDriverEntryPoint, so the
// extension needs no link against libcuda.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

namespace dtb {

namespace {

struct VmmApi {
  CUresult (*getGranularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
  CUresult (*create)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long);
  CUresult (*exportHandle)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType, unsigned long long);
  CUresult (*importHandle)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  CUresult (*reserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  CUresult (*setAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);
  CUresult (*unmap)(CUdeviceptr, size_t);
  CUresult (*addressFree)(CUdeviceptr, size_t);
  CUresult (*release)(CUmemGenericAllocationHandle);
  // switch multicast (NVLS)
  CUresult (*deviceGet)(CUdevice*, int);
  CUresult (*deviceGetAttribute)(int*, CUdevice_attribute, CUdevice);
  CUresult (*mcGranularity)(size_t*, const CUmulticastObjectProp*, CUmulticastGranularity_flags);
  CUresult (*mcCreate)(CUmemGenericAllocationHandle*, const CUmulticastObjectProp*);
  CUresult (*mcAddDevice)(CUmemGenericAllocationHandle, CUdevice);
  CUresult (*mcBindMem)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle, size_t, size_t,
                        unsigned long long);
  CUresult (*mcUnbind)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t);
};

template <typename F>
void resolve(F& fn, const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  const cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p, "vmm: driver entry point ", name,
              " unavailable");
  fn = reinterpret_cast<F>(p);
}

const VmmApi& api() {
  static VmmApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    resolve(a.getGranularity, "cuMemGetAllocationGranularity");
    resolve(a.create, "cuMemCreate");
    resolve(a.exportHandle, "cuMemExportToShareableHandle");
    resolve(a.importHandle, "cuMemImportFromShareableHandle");
    resolve(a.reserve, "cuMemAddressReserve");
    resolve(a.map, "cuMemMap");
    resolve(a.setAccess, "cuMemSetAccess");
    resolve(a.unmap, "cuMemUnmap");
    resolve(a.addressFree, "cuMemAddressFree");
    resolve(a.release, "cuMemRelease");
    resolve(a.deviceGet, "cuDeviceGet");
    resolve(a.deviceGetAttribute, "cuDeviceGetAttribute");
    resolve(a.mcGranularity, "cuMulticastGetGranularity");
    resolve(a.mcCreate, "cuMulticastCreate");
    resolve(a.mcAddDevice, "cuMulticastAddDevice");
    resolve(a.mcBindMem, "cuMulticastBindMem");
    resolve(a.mcUnbind, "cuMulticastUnbind");
  });
  return a;
}

#define DTB_CU(call, what)                                                      \
  do {                                                                          \
    const CUresult r_ = (call);                                                 \
    TORCH_CHECK(r_ == CUDA_SUCCESS, "vmm: ", what, " failed with code ", (int)r_); \
  } while (0)

CUmemAllocationProp device_prop(int dev) {
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = dev;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return prop;
}

struct Mapping {
  CUmemGenericAllocationHandle handle;
  size_t size;
};
std::mutex g_mu;
std::map<int64_t, Mapping> g_maps;  // mapped base address -> handle and size

// Reserve an address range for `handle` and map it read/write for device `dev`.
int64_t map_handle(CUmemGenericAllocationHandle h, size_t size, size_t gran, int dev) {
  const VmmApi& A = api();
  CUdeviceptr va = 0;
  DTB_CU(A.reserve(&va, size, gran, 0, 0), "cuMemAddressReserve");
  CUresult r = A.map(va, size, 0, h, 0);
  if (r != CUDA_SUCCESS) {
    A.addressFree(va, size);
    TORCH_CHECK(false, "vmm: cuMemMap failed with code ", (int)r);
  }
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = dev;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = A.setAccess(va, size, &acc, 1);
  if (r != CUDA_SUCCESS) {
    A.unmap(va, size);
    A.addressFree(va, size);
    TORCH_CHECK(false, "vmm: cuMemSetAccess failed with code ", (int)r);
  }
  std::lock_guard<std::mutex> g(g_mu);
  g_maps[(int64_t)va] = {h, size};
  return (int64_t)va;
}

size_t granularity(int dev) {
  const CUmemAllocationProp prop = device_prop(dev);
  size_t g = 0;
  DTB_CU(api().getGranularity(&g, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "cuMemGetAllocationGranularity");
  return g ? g : ((size_t)2 << 20);
}

}  // namespace

// Zero-filled device memory of at least `nbytes` on the current device, exportable as a
// file descriptor.  Returns (address, descriptor, mapped size).  The caller owns the
// descriptor (close it once every peer has received it).
std::tuple<int64_t, int64_t, int64_t> vmm_alloc(int64_t nbytes) {
  TORCH_CHECK(nbytes > 0, "vmm_alloc: size must be positive");
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  cudaFree(nullptr);  // make sure the primary context exists and is current
  const VmmApi& A = api();
  const size_t gran = granularity(dev);
  const size_t size = ((size_t)nbytes + gran - 1) / gran * gran;
  const CUmemAllocationProp prop = device_prop(dev);
  CUmemGenericAllocationHandle h;
  DTB_CU(A.create(&h, size, &prop, 0), "cuMemCreate");
  int64_t va = 0;
  try {
    va = map_handle(h, size, gran, dev);
  } catch (...) {
    A.release(h);
    throw;
  }
  C10_CUDA_CHECK(cudaMemset(reinterpret_cast<void*>(va), 0, size));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  int fd = -1;
  DTB_CU(A.exportHandle(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0), "cuMemExportToShareableHandle");
  return {va, (int64_t)fd, (int64_t)size};
}

// Map a peer's allocation, received as a file descriptor, for the current device.  The
// descriptor may be closed after this returns.  Returns the local address.
int64_t vmm_import(int64_t fd, int64_t size) {
  TORCH_CHECK(fd >= 0 && size > 0, "vmm_import: bad descriptor or size");
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  cudaFree(nullptr);
  const VmmApi& A = api();
  const size_t gran = granularity(dev);
  TORCH_CHECK((size_t)size % gran == 0, "vmm_import: size is not a multiple of the allocation granularity");
  CUmemGenericAllocationHandle h;
  DTB_CU(A.importHandle(&h, reinterpret_cast<void*>((uintptr_t)fd), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
         "cuMemImportFromShareableHandle");
  try {
    return map_handle(h, (size_t)size, gran, dev);
  } catch (...) {
    A.release(h);
    throw;
  }
}

// Unmap an address returned by vmm_alloc / vmm_import and drop this process's
// reference to the physical memory (it is freed when the last process lets go).
void vmm_free(int64_t va) {
  Mapping m;
  {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_maps.find(va);
    TORCH_CHECK(it != g_maps.end(), "vmm_free: unknown address");
    m = it->second;
    g_maps.erase(it);
  }
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  const VmmApi& A = api();
  A.unmap((CUdeviceptr)va, m.size);
  A.addressFree((CUdeviceptr)va, m.size);
  A.release(m.handle);
}

// ---------------------------------------------------------------- NVSwitch multicast
// A multicast object spans one VMM allocation on every rank: a store through its
// mapping (multimem.st) lands in every rank's allocation, and a multimem.ld_reduce
// through it returns the sum over ranks, computed in the switch.  Rank 0 creates the
// object and passes it to the others as a file descriptor; every rank adds its own
// device, binds its allocation (the driver blocks the bind until all devices have
// been added) and maps the object into its address space.
//
// Teardown rule: every rank must have finished its multimem work before any rank
// unbinds (NVLinkGroup.close() synchronises and barriers first).  A process that
// dies with memory still bound can disturb the other ranks' GPUs, so code that
// runs these collectives never exits a rank on purpose while the binding exists.

namespace {
struct McMapping {
  CUmemGenericAllocationHandle mc;
  size_t size;
  CUdevice dev;
  bool bound;
};
std::map<int64_t, McMapping> g_mc;  // multicast mapping address -> object, size, device

CUmulticastObjectProp mc_prop(int64_t size, int64_t ndev) {
  CUmulticastObjectProp prop = {};
  prop.numDevices = (unsigned)ndev;
  prop.size = (size_t)size;
  prop.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  prop.flags = 0;
  return prop;
}

CUdevice current_cu_device() {
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  cudaFree(nullptr);
  CUdevice d;
  DTB_CU(api().deviceGet(&d, dev), "cuDeviceGet");
  return d;
}
}  // namespace

// Whether the current device supports switch multicast and reductions.
bool mc_supported() {
  const CUdevice d = current_cu_device();
  int v = 0;
  if (api().deviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d) != CUDA_SUCCESS) return false;
  return v != 0;
}

// Size granule of a multicast object of `ndev` devices (also a multiple of the VMM
// allocation granularity, so one VMM allocation of this size can be bound whole).
int64_t mc_granularity(int64_t ndev) {
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  const CUmulticastObjectProp prop = mc_prop(1, ndev);
  size_t g = 0;
  DTB_CU(api().mcGranularity(&g, &prop, CU_MULTICAST_GRANULARITY_MINIMUM), "cuMulticastGetGranularity");
  const size_t vg = granularity(dev);
  size_t m = std::max(g, vg);
  if (m % g || m % vg) m = g * vg;  // both are powers of two in practice; keep a common multiple regardless
  return (int64_t)m;
}

// Creates a multicast object of `size` bytes for `ndev` devices; returns (handle, fd).
// The caller passes the descriptor to the other ranks and closes it.
std::tuple<int64_t, int64_t> mc_create(int64_t size, int64_t ndev) {
  TORCH_CHECK(size > 0 && ndev >= 2, "mc_create: positive size and at least two devices");
  current_cu_device();
  const CUmulticastObjectProp prop = mc_prop(size, ndev);
  CUmemGenericAllocationHandle h;
  DTB_CU(api().mcCreate(&h, &prop), "cuMulticastCreate");
  int fd = -1;
  const CUresult r = api().exportHandle(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) {
    api().release(h);
    TORCH_CHECK(false, "vmm: exporting the multicast object failed with code ", (int)r);
  }
  return {(int64_t)h, (int64_t)fd};
}

// Imports a multicast object received as a file descriptor (which may then be closed).
int64_t mc_import(int64_t fd) {
  TORCH_CHECK(fd >= 0, "mc_import: bad descriptor");
  current_cu_device();
  CUmemGenericAllocationHandle h;
  DTB_CU(api().importHandle(&h, reinterpret_cast<void*>((uintptr_t)fd), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
         "cuMemImportFromShareableHandle (multicast)");
  return (int64_t)h;
}

// Adds the current device to multicast object `mc`.  Every rank must have done so
// before any rank binds memory (the driver blocks a bind until the whole team has
// joined), so the caller confirms that all ranks joined - over the host - before it
// calls mc_bind_map; on failure it releases the object with mc_release.
void mc_add_device(int64_t mc) {
  const CUresult r = api().mcAddDevice((CUmemGenericAllocationHandle)mc, current_cu_device());
  TORCH_CHECK(r == CUDA_SUCCESS, "vmm: cuMulticastAddDevice failed with code ", (int)r);
}

// Drops this process's reference to a multicast object that was never mapped.
void mc_release(int64_t mc) { api().release((CUmemGenericAllocationHandle)mc); }

// Binds this rank's VMM allocation `local_va` (from vmm_alloc, `size` bytes) to
// multicast object `mc` (which every rank has joined, see mc_add_device) and maps the
// object (made for `ndev` devices) for the current device.  Returns the multicast
// address: multimem instructions on it reach every rank's allocation at the same
// offset.  On failure the object is released.
int64_t mc_bind_map(int64_t mc, int64_t local_va, int64_t size, int64_t ndev) {
  const VmmApi& A = api();
  const CUmemGenericAllocationHandle h = (CUmemGenericAllocationHandle)mc;
  Mapping local;
  {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_maps.find(local_va);
    if (it == g_maps.end() || it->second.size < (size_t)size) {
      A.release(h);
      TORCH_CHECK(false, "mc_bind_map: the local buffer is not a vmm_alloc allocation of at least ", size, " bytes");
    }
    local = it->second;
  }
  const CUdevice d = current_cu_device();
  CUresult r = A.mcBindMem(h, 0, local.handle, 0, (size_t)size, 0);
  if (r != CUDA_SUCCESS) {
    A.release(h);
    TORCH_CHECK(false, "vmm: cuMulticastBindMem failed with code ", (int)r);
  }
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  CUdeviceptr va = 0;
  r = A.reserve(&va, (size_t)size, (size_t)mc_granularity(ndev), 0, 0);
  if (r == CUDA_SUCCESS) r = A.map(va, (size_t)size, 0, h, 0);
  if (r == CUDA_SUCCESS) {
    CUmemAccessDesc acc = {};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = dev;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    r = A.setAccess(va, (size_t)size, &acc, 1);
    if (r != CUDA_SUCCESS) A.unmap(va, (size_t)size);
  }
  if (r != CUDA_SUCCESS) {
    if (va) A.addressFree(va, (size_t)size);
    A.mcUnbind(h, d, 0, (size_t)size);
    A.release(h);
    TORCH_CHECK(false, "vmm: mapping the multicast object failed with code ", (int)r);
  }
  std::lock_guard<std::mutex> g(g_mu);
  g_mc[(int64_t)va] = {h, (size_t)size, d, true};
  return (int64_t)va;
}

// Unmaps a multicast address from mc_bind_map, unbinds this rank's memory and drops
// this process's reference to the object.  Every rank's multimem work on it must be
// finished (the caller synchronises and barriers across ranks first).
void mc_free(int64_t mc_va) {
  McMapping m;
  {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_mc.find(mc_va);
    TORCH_CHECK(it != g_mc.end(), "mc_free: unknown multicast address");
    m = it->second;
    g_mc.erase(it);
  }
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  const VmmApi& A = api();
  A.unmap((CUdeviceptr)mc_va, m.size);
  A.addressFree((CUdeviceptr)mc_va, m.size);
  if (m.bound) A.mcUnbind(m.mc, m.dev, 0, m.size);
  A.release(m.mc);
}

}  // namespace dtb
