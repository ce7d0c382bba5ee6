// cottus::PageTable — same interface and exceptions as the reference
// (page_table.h:9-14, page_table.cpp:7-38): an append-only logical->physical
// block list; getBlock/operator[] throw std::out_of_range outside [0, n).
#pragma once

#include <cstdint>
#include <vector>

namespace cottus {

class PageTable {
public:
    explicit PageTable(int32_t blockSize);  // std::invalid_argument if blockSize <= 0
    void appendBlock(int32_t blockId);
    int32_t getBlock(int32_t logicalIndex) const;
    int32_t operator[](int32_t logicalIndex) const;
    int32_t numBlocks() const;
    int32_t blockSize() const;
    const int32_t* data() const { return blocks_.data(); }

private:
    std::vector<int32_t> blocks_;
    int32_t blockSize_;
};

}  // namespace cottus
