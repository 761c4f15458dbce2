// Host-memory segments shared by the ranks of one box; see host_segment.hpp.
#include "host_segment.hpp"

#include <cerrno>
#include <cstring>
#include <stdexcept>

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace ep {

namespace {

std::string errno_text(const char* what, const std::string& name) {
    return std::string("HostSegment ") + what + " '" + name + "': " + std::strerror(errno);
}

}  // namespace

HostSegment::HostSegment(const std::string& name, int64_t bytes, bool create) : name_(name), bytes_(bytes), owner_(create) {
    TORCH_CHECK(!name.empty() && name[0] == '/' && name.find('/', 1) == std::string::npos,
                "HostSegment: the name must be '/' followed by no further '/'");
    TORCH_CHECK(bytes > 0, "HostSegment: bytes must be positive");
    const int fd = create ? shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600) : shm_open(name.c_str(), O_RDWR, 0);
    if (fd < 0) throw std::runtime_error(errno_text(create ? "create" : "open", name));
    if (create && ftruncate(fd, (off_t)bytes) != 0) {
        const std::string msg = errno_text("resize", name);
        close(fd);
        shm_unlink(name.c_str());
        throw std::runtime_error(msg);
    }
    if (!create) {
        struct stat st {};
        if (fstat(fd, &st) != 0 || (int64_t)st.st_size < bytes) {
            close(fd);
            throw std::runtime_error("HostSegment open '" + name + "': smaller than the requested size");
        }
    }
    void* p = mmap(nullptr, (size_t)bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);  // the mapping keeps the object alive
    if (p == MAP_FAILED) {
        const std::string msg = errno_text("map", name);
        if (create) shm_unlink(name.c_str());
        throw std::runtime_error(msg);
    }
    base_ = p;
}

HostSegment::~HostSegment() {
    try {
        destroy();
    } catch (...) {
    }
}

int64_t HostSegment::device_ptr() {
    TORCH_CHECK(!destroyed_, "HostSegment was destroyed");
    if (!registered_) {
        cudaError_t e = cudaHostRegister(base_, (size_t)bytes_, cudaHostRegisterMapped | cudaHostRegisterPortable);
        TORCH_CHECK(e == cudaSuccess, "HostSegment: cudaHostRegister failed: ", cudaGetErrorString(e));
        e = cudaHostGetDevicePointer(&dev_, base_, 0);
        if (e != cudaSuccess) {
            cudaHostUnregister(base_);
            TORCH_CHECK(false, "HostSegment: cudaHostGetDevicePointer failed: ", cudaGetErrorString(e));
        }
        registered_ = true;
    }
    return reinterpret_cast<int64_t>(dev_);
}

torch::Tensor HostSegment::host_view(int64_t offset, int64_t bytes) const {
    TORCH_CHECK(!destroyed_, "HostSegment was destroyed");
    TORCH_CHECK(offset >= 0 && bytes >= 0 && offset + bytes <= bytes_, "HostSegment view out of range");
    return torch::from_blob(static_cast<uint8_t*>(base_) + offset, {bytes}, torch::dtype(torch::kUInt8));
}

void HostSegment::destroy() {
    if (destroyed_) return;
    destroyed_ = true;
    if (registered_) {
        cudaDeviceSynchronize();  // no kernel still reads the mapping
        cudaHostUnregister(base_);
        registered_ = false;
    }
    if (base_ != nullptr) munmap(base_, (size_t)bytes_);
    base_ = nullptr;
    if (owner_) shm_unlink(name_.c_str());
}

}  // namespace ep
