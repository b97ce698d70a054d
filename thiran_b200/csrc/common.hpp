// Shared host-side types of the B200 engine: failures, dtypes, helpers.
#pragma once

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#include "thiran_b200.h"

namespace thb {

// A failure carries the C-ABI status plus a code such as GPU-INPUT-ARITY or a
// semantic failure id such as TH-SPEC-I64-OVERFLOW. The categories follow
// GpuErrorCategory (include/backend/v0/NativeGpu.hpp:21-28).
enum class Category { Validation, BackendUnavailable, InvalidDevice, Unsupported, Runtime, Semantic };

class Failure : public std::exception {
public:
    Failure(Category category, std::string code, std::string message)
        : category_(category), code_(std::move(code)), message_(std::move(message)) {}
    const char* what() const noexcept override { return message_.c_str(); }
    Category category() const noexcept { return category_; }
    const std::string& code() const noexcept { return code_; }
    const std::string& message() const noexcept { return message_; }
    int status() const noexcept {
        switch (category_) {
        case Category::Semantic: return THB_STATUS_SEMANTIC;
        case Category::Validation:
        case Category::Unsupported: return THB_STATUS_ABI;
        default: return THB_STATUS_BACKEND;
        }
    }
    // Text written into the caller's failure buffer.
    std::string text() const {
        if (category_ == Category::Semantic) return code_;
        return code_ + ": " + message_;
    }
private:
    Category category_;
    std::string code_;
    std::string message_;
};

[[noreturn]] inline void fail(Category category, const std::string& code, const std::string& message) {
    throw Failure(category, code, message);
}

enum class DType : std::uint32_t { I64 = THB_DTYPE_I64, F32 = THB_DTYPE_F32, BF16 = THB_DTYPE_BF16 };

inline std::size_t width(DType dtype) {
    switch (dtype) {
    case DType::I64: return 8;
    case DType::F32: return 4;
    case DType::BF16: return 2;
    }
    return 0;
}

inline const char* dtypeName(DType dtype) {
    switch (dtype) {
    case DType::I64: return "i64";
    case DType::F32: return "f32";
    case DType::BF16: return "bf16";
    }
    return "?";
}

inline void writeText(char* buffer, std::uint64_t capacity, const std::string& text) {
    if (!buffer || capacity == 0) return;
    const std::size_t n = text.size() < capacity - 1 ? text.size() : static_cast<std::size_t>(capacity - 1);
    std::memcpy(buffer, text.data(), n);
    buffer[n] = '\0';
}

// Overflow-checked size arithmetic (the storage::checkedMultiply contract,
// include/storage/v0/Storage.hpp:51-55).
inline std::uint64_t checkedMul(std::uint64_t a, std::uint64_t b) {
    std::uint64_t r = 0;
    if (__builtin_mul_overflow(a, b, &r)) fail(Category::Validation, "GPU-SIZE-OVERFLOW", "element count overflows u64");
    return r;
}

} // namespace thb
