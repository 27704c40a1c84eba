// Tiling constants shared by the read kernels.
#pragma once

namespace mom {
constexpr int kReadThreads = 256;   // 8 warps x 16 rows = one 128-token tile
constexpr int kDkvThreads = 128;    // dK/dV kernel: 4 warps x 16 slots
constexpr int kDkvSub = 64;         // dK/dV kernel: tokens per compute sub-tile
constexpr int kSlotChunk = 64;      // slots per K/V pipeline step
}  // namespace mom
