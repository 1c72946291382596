// bpe_tokenizer.h - the byte-level BPE text tokenizer of a qwen3 GGUF (host).
//
// Behaviour follows the reference tokenizer (bnn-sw-v2/tokenizer/
// tokenizer-bpe.c), the one behind BNNE_Tokenize / BNNE_TokenPiece /
// BNNE_TokenIsEog (bnn-sw-v2/bnn-engine.h:106-116):
//   - GPT-2 byte-to-code-point table: bytes 33..126, 161..172, 174..255 map to
//     themselves, the other 68 bytes to 256, 257, ... in byte order
//     (tokenizer-bpe.c:718-733); every byte's symbol must be a token;
//   - special tokens are the tokens of type 3 (control) and 4 (user defined);
//     with parse_special they are matched as literals, longest first, lowest
//     id among equal lengths, scanning byte by byte (tokenizer-bpe.c:548-582);
//   - the text between specials must be valid UTF-8 (RFC 3629; no overlongs,
//     surrogates or code points above U+10FFFF), else the call fails with
//     EINVAL keeping the ids already produced;
//   - the Qwen2 pre-tokenizer split (tokenizer-bpe.c:418-538);
//   - BPE over each chunk: repeatedly merge the adjacent pair of lowest merge
//     rank, leftmost among equals (tokenizer-bpe.c:346-373); a final symbol
//     that is not a token becomes the byte tokens of its bytes;
//   - duplicate token strings: the last id wins; duplicate merges: the first
//     rank wins; merge lines without an inner space or with an empty side
//     are skipped but keep their line number as rank;
//   - pieces: control/user-defined tokens verbatim, others mapped back through
//     the byte table (tokenizer-bpe.c:592-633); EOG ids: eos_token_id and the
//     tokens "<|endoftext|>" and "<|im_end|>", eight at most.
// The implementation is this project's own: symbols are interned strings,
// merges a (left, right) symbol-pair table, and each chunk's merges run on a
// linked list with a min-heap of candidate pairs, O(n log n) per chunk.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace bnn {

class GgufFile;

enum class TokStatus { kOk = 0, kInvalid, kRange, kFormat };

class BpeTokenizer {
  public:
    // Reads tokenizer.ggml.{tokens,token_type,merges,eos_token_id}. kFormat
    // (with *why) for a missing vocabulary or byte token, kRange for a
    // vocabulary above 2^32 - 1 entries.
    TokStatus build(const GgufFile& g, std::string* why);

    // Encodes len bytes of text. *count receives the ids written, also on
    // failure: kRange when capacity ran out (ids[0..capacity) written),
    // kInvalid for text that is not valid UTF-8 outside special tokens.
    TokStatus encode(const char* text, size_t len, bool parse_special, int32_t* ids, uint32_t capacity,
                     uint32_t* count) const;

    // The decoded bytes of token id (NUL-terminated, owned by this object);
    // kRange for an id outside the vocabulary.
    TokStatus piece(int32_t id, const char** bytes, size_t* len) const;

    bool is_eog(int32_t id) const;
    uint32_t size() const { return n_tokens_; }

  private:
    struct Merge {
        uint32_t rank;
        uint32_t result;  // symbol of left + right
    };
    struct Special {
        uint32_t id;
        uint32_t off, len;  // in vocab_
    };
    struct Scratch;

    bool encode_segment(const uint8_t* text, size_t len, Scratch& w) const;
    void encode_chunk(const uint8_t* text, size_t len, Scratch& w) const;
    const Special* match_special(const uint8_t* text, size_t left) const;

    uint32_t n_tokens_ = 0;
    std::string vocab_;               // token strings back to back
    std::vector<uint32_t> vocab_off_;  // [n_tokens_ + 1]
    std::string pieces_;              // decoded pieces, each followed by NUL
    std::vector<uint32_t> piece_off_;  // [n_tokens_ + 1] (lengths exclude the NUL)
    std::vector<int32_t> sym_token_;   // symbol -> token id (last duplicate), -1 if none
    std::unordered_map<uint64_t, Merge> merges_;  // (left symbol << 32 | right symbol)
    uint32_t byte_sym_[256] = {};
    int32_t byte_token_[256] = {};
    std::vector<Special> specials_;                // id order
    std::vector<uint32_t> special_by_byte_[256];  // indexes into specials_, longest first
    int32_t empty_special_ = -1;                   // first special with an empty text
    uint32_t eog_[8] = {};
    uint32_t n_eog_ = 0;
};

}  // namespace bnn
