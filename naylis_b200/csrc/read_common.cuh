// Tiling constants shared by the read kernels.
#pragma once

namespace mom {
constexpr int kReadThreads = 128;   // 4 warps x 16 rows
constexpr int kSlotChunk = 64;      // slots per K/V pipeline step
}  // namespace mom
