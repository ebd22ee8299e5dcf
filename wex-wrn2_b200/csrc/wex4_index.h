// The expert records of a validated WEX4 index, for readers that fetch records from a file
// themselves (file_stream.cpp). Implemented in wex4_api.cpp with the container rules it applies to
// every other entry point (c/wex4.h:185-437).
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include "wex_entry.h"

namespace wexb {

struct FileExpert {
    uint32_t owner;        // layer << 16 | expert
    uint32_t codec;        // 0 RAW or 5 WNR3
    uint32_t stored;       // stored bytes at entry.file_offset
    uint32_t model;        // WNR3: the id of its WNM2 blob, else 0
    bool value_exact;      // the record's VALUE_EXACT flag (WNR3 only)
    uint8_t sha[32];       // SHA-256 of the stored bytes, from the index
    WexEntry entry;        // the 72-byte legacy entry rebuilt from the index (c/wex4.h:264-290)
};
struct FileModel {         // a WNM2 blob
    uint64_t offset, bytes;
    uint32_t id;
    uint8_t sha[32];
};
struct FileIndex {
    uint64_t file_bytes = 0, index_offset = 0, index_len = 0;
    uint32_t layers = 0, experts = 0;
    std::vector<FileExpert> records;   // the EXPERT records, in record order
    std::vector<FileModel> models;
};

// The header page: 0 and the index position and length (page-aligned), or a WEX4_E_* code.
int file_header(const uint8_t *page, uint64_t file_bytes, FileIndex *out);
// The index (index_len bytes, as file_header gave): 0 and out->records / out->models, or a WEX4_E_* code.
// Expert records of codecs other than RAW and WNR3 are refused with WEX4_E_UNSUPPORTED.
int file_index(const uint8_t *page, const uint8_t *index, FileIndex *out);
// FIPS 180-4 SHA-256 on the host.
void host_sha256(const uint8_t *p, size_t n, uint8_t out[32]);

}  // namespace wexb
