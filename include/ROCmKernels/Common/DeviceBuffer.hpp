// Owning device allocation. Same interface as ROCmKernels.Common/include/ROCmKernels/Common/DeviceBuffer.hpp:15-101
// (Resize, Release, CopyFromHost, CopyToHost, Data, Count, ByteSize; move-only), over the CUDA runtime.
#pragma once

#include <ROCmKernels/Common/Error.hpp>

#include <cstddef>
#include <stdexcept>
#include <utility>

namespace ROCmKernels {
    template <typename T> class DeviceBuffer {
        T *m_pData = nullptr;
        std::size_t m_elementCount = 0;

        void CheckCount(std::size_t elementCount) const {
            if (elementCount > this->m_elementCount) throw std::out_of_range("DeviceBuffer transfer larger than the allocation");
        }

      public:
        DeviceBuffer() = default;
        explicit DeviceBuffer(std::size_t elementCount) { this->Resize(elementCount); }
        ~DeviceBuffer() {
            if (this->m_pData != nullptr) (void)cudaFree(this->m_pData);
        }

        DeviceBuffer(const DeviceBuffer &) = delete;
        DeviceBuffer &operator=(const DeviceBuffer &) = delete;
        DeviceBuffer(DeviceBuffer &&other) noexcept
            : m_pData(std::exchange(other.m_pData, nullptr)), m_elementCount(std::exchange(other.m_elementCount, 0)) {}
        DeviceBuffer &operator=(DeviceBuffer &&other) noexcept {
            if (this != &other) {
                if (this->m_pData != nullptr) (void)cudaFree(this->m_pData);
                this->m_pData = std::exchange(other.m_pData, nullptr);
                this->m_elementCount = std::exchange(other.m_elementCount, 0);
            }
            return *this;
        }

        /// Replaces the allocation with room for elementCount elements (contents undefined).
        void Resize(std::size_t elementCount) {
            this->Release();
            if (elementCount == 0) return;
            ROCMKERNELS_HIP_CHECK(cudaMalloc(reinterpret_cast<void **>(&this->m_pData), elementCount * sizeof(T)));
            this->m_elementCount = elementCount;
        }

        void Release() {
            if (this->m_pData != nullptr) {
                T *pointer = std::exchange(this->m_pData, nullptr);
                ROCMKERNELS_HIP_CHECK(cudaFree(pointer));
            }
            this->m_elementCount = 0;
        }

        /// Synchronous copy when stream is null, otherwise ordered on stream.
        void CopyFromHost(const T *source, std::size_t elementCount, hipStream_t stream = nullptr) {
            this->CheckCount(elementCount);
            if (elementCount == 0) return;
            if (stream == nullptr)
                ROCMKERNELS_HIP_CHECK(cudaMemcpy(this->m_pData, source, elementCount * sizeof(T), cudaMemcpyHostToDevice));
            else
                ROCMKERNELS_HIP_CHECK(cudaMemcpyAsync(this->m_pData, source, elementCount * sizeof(T), cudaMemcpyHostToDevice, stream));
        }

        void CopyToHost(T *destination, std::size_t elementCount, hipStream_t stream = nullptr) const {
            this->CheckCount(elementCount);
            if (elementCount == 0) return;
            if (stream == nullptr)
                ROCMKERNELS_HIP_CHECK(cudaMemcpy(destination, this->m_pData, elementCount * sizeof(T), cudaMemcpyDeviceToHost));
            else
                ROCMKERNELS_HIP_CHECK(cudaMemcpyAsync(destination, this->m_pData, elementCount * sizeof(T), cudaMemcpyDeviceToHost, stream));
        }

        [[nodiscard]] T *Data() const noexcept { return this->m_pData; }
        [[nodiscard]] std::size_t Count() const noexcept { return this->m_elementCount; }
        [[nodiscard]] std::size_t ByteSize() const noexcept { return this->m_elementCount * sizeof(T); }
    };
} // namespace ROCmKernels
