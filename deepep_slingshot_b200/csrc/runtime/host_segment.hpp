// Host-memory segments shared by the ranks of one box (the elastic API's hybrid CPU memory).
//
// The reference allocates a CPU segment per rank, exchanges POSIX handles for it and keeps its
// Engram storage there ([DE]deep_ep/buffers/elastic.py:208-213, `create_cpu_handle`;
// [DE]csrc/kernels/backend/symmetric.hpp:72-322). Here every rank creates one named POSIX
// shared-memory object (`shm_open` + `mmap`), the names are exchanged over torch.distributed, and
// every rank maps every rank's segment. For GPU access a process registers each mapping with CUDA
// (`cudaHostRegister`, mapped + portable) and its kernels read the rows through the device pointer
// (PCIe / C2C, no copy engine). The creator unlinks the name when it is destroyed; the memory stays
// valid for the ranks that still map it until they unmap.
#pragma once

#include <torch/extension.h>

#include <cstdint>
#include <string>

namespace ep {

class HostSegment {
public:
    // `create`: make a new object of `bytes` (fails if the name exists); otherwise open an existing one.
    HostSegment(const std::string& name, int64_t bytes, bool create);
    ~HostSegment();
    HostSegment(const HostSegment&) = delete;
    HostSegment& operator=(const HostSegment&) = delete;

    const std::string& name() const { return name_; }
    int64_t bytes() const { return bytes_; }
    bool is_owner() const { return owner_; }
    int64_t host_ptr() const { return reinterpret_cast<int64_t>(base_); }
    // Registers the mapping with CUDA on first use (current device) and returns its device pointer.
    int64_t device_ptr();
    // CPU uint8 view of [offset, offset + bytes) of the mapping (shares its memory).
    torch::Tensor host_view(int64_t offset, int64_t bytes) const;
    void destroy();

private:
    std::string name_;
    int64_t bytes_ = 0;
    bool owner_ = false, registered_ = false, destroyed_ = false;
    void* base_ = nullptr;
    void* dev_ = nullptr;
};

}  // namespace ep
