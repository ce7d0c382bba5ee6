// cottus::BlockAllocator — same interface and exceptions as the reference
// (block_allocator.h:9-14, block_allocator.cpp:7-55): fixed pool, LIFO free
// list whose first allocation is block 0; "Out of memory" / "Invalid block
// ID" / "Double free detected" errors.
#pragma once

#include <cstdint>
#include <vector>

namespace cottus {

class BlockAllocator {
public:
    BlockAllocator(int32_t totalBlocks, int32_t blockSize);
    int32_t allocateBlock();            // std::runtime_error("Out of memory: no free blocks")
    void freeBlock(int32_t blockId);    // std::invalid_argument / std::runtime_error (double free)
    int32_t numFreeBlocks() const;
    int32_t totalBlocks() const;
    int32_t blockSize() const;

private:
    int32_t total_;
    int32_t blockSize_;
    std::vector<int32_t> freeStack_;
    std::vector<uint8_t> inUse_;
};

}  // namespace cottus
