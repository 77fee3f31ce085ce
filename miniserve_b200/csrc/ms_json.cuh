// JSON-grammar allowed-token mask: allowed[t] = is_valid_prefix(prefix + vocab[t])
// for miniserve's JSONLogitsProcessor.is_valid_prefix (miniserve/sampler.py:
// 139-148), i.e. "the text is empty, starts with '{', parses with json.loads,
// or json.loads fails with an 'Expecting ...' / 'Unterminated ...' error".
//
// A byte-streaming automaton decides that class.  It follows the order in
// which CPython 3.12's json C scanner reports errors: the first error decides
// ("Invalid \\escape", "Invalid \\uXXXX escape", "Invalid control character"
// and "Extra data" are the False classes); an integer of more than 4300 digits
// or 9997 nested containers makes the reference raise instead (RAISE here).
// The scanner's one-character lookaheads (a '.' or 'e' that only belongs to a
// number when a digit follows, a literal that must be present in full, a
// \uXXXX escape that needs one more character after its digits) are pending
// states resolved by the next byte or by the end of the text.
//
// Row state (kJsonStateWords 32-bit words, in HBM between calls): a JState
// header and the container stack, one bit per level (1 = object).
#pragma once

#include "ms_common.cuh"

namespace ms {

constexpr int kJsonThreads = 256;
constexpr int kJsonMaxDepth = 9996;                       // the 9997th nested container raises
constexpr int kJsonStackWords = (kJsonMaxDepth + 31) / 32;
constexpr int kJsonHeaderWords = 4;
constexpr int kJsonStateWords = 320;                      // header + stack, padded
constexpr uint32_t kJsonIntDigits = 4300;
static_assert(kJsonHeaderWords + kJsonStackWords <= kJsonStateWords, "state layout");

enum : uint8_t { J_UNDECIDED = 0, J_TRUE = 1, J_FALSE = 2, J_RAISE = 3 };
enum : uint8_t {
  JM_TOP = 0,    // before the top-level value
  JM_VALUE,      // a value expected (after ',' in an array, ':' in an object)
  JM_ARR_FIRST,  // after '[': ']' closes the empty array
  JM_OBJ_FIRST,  // after '{': '}' closes the empty object, '"' opens a key
  JM_OBJ_KEY,    // after ',' in an object: '"' opens a key
  JM_AFTER_KEY,  // a key read: ':' expected
  JM_AFTER,      // a value read
  JM_STR,        // string body (key: an object key)
  JM_ESC,        // after a backslash
  JM_UHEX,       // inside \uXXXX (aux = digits read)
  JM_UDONE,      // four digits read: one more character must follow
  JM_NUM,        // number (sub = phase)
  JM_LIT         // literal (sub = which, aux = characters matched)
};
enum : uint8_t { NP_MINUS = 0, NP_ZERO, NP_INT, NP_DOT, NP_FRAC, NP_E, NP_ESIGN, NP_EXP };

struct JState {
  uint8_t decided, mode, sub, aux;
  uint8_t key, first, isfloat, pad;  // first: 1 once the text has a character
  int32_t depth;
  uint32_t ndig;  // integer digits of the current number (saturates)
};
static_assert(sizeof(JState) == 16, "JState is four words");

// null true false NaN Infinity -Infinity
__host__ __device__ __forceinline__ char j_lit_char(int id, int i) {
  return id == 0 ? "null"[i] : id == 1 ? "true"[i] : id == 2 ? "false"[i] : id == 3 ? "NaN"[i]
       : id == 4 ? "Infinity"[i] : "-Infinity"[i];
}
__host__ __device__ __forceinline__ int j_lit_len(int id) {
  return id == 0 || id == 1 ? 4 : id == 2 ? 5 : id == 3 ? 3 : id == 4 ? 8 : 9;
}
__host__ __device__ __forceinline__ bool j_ws(uint8_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
__host__ __device__ __forceinline__ bool j_digit(uint8_t c) { return c >= '0' && c <= '9'; }
__host__ __device__ __forceinline__ bool j_hex(uint8_t c) {
  return j_digit(c) || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F');
}

// Container stacks: push(level, is_object) when a container opens at
// `level`, pop(level) when the container at `level` closes, is_obj(level).
//
// The stack of one row in global memory (feeding the prefix).
struct JStackGlobal {
  uint32_t *bits;
  __host__ __device__ bool is_obj(int level) const { return (bits[level >> 5] >> (level & 31)) & 1u; }
  __host__ __device__ void push(int level, bool obj) {
    const uint32_t m = 1u << (level & 31);
    bits[level >> 5] = obj ? (bits[level >> 5] | m) : (bits[level >> 5] & ~m);
  }
  __host__ __device__ void pop(int) {}
};

// The stack seen by one token continuing a row: the row's levels (shared
// memory, read only) below the lowest depth the token has popped to, and the
// levels the token opened itself in a 128-level register window starting 64
// below the row's depth.  A token that closes more than 64 of the row's
// containers and then opens one, or opens more than 64 beyond them, sets
// `over` (its answer is not computed).
struct JStackTok {
  const uint32_t *bits;
  int w0;        // first level of the window
  int floor_;    // lowest depth the token popped to
  bool over;
  unsigned long long lo, hi;  // levels w0 .. w0+63, w0+64 .. w0+127
  __host__ __device__ JStackTok(const uint32_t *b, int depth)
      : bits(b), w0(depth - 64), floor_(depth), over(false), lo(0ull), hi(0ull) {}
  __host__ __device__ bool is_obj(int level) const {
    if (level < floor_) return (bits[level >> 5] >> (level & 31)) & 1u;
    const int i = level - w0;
    if (i < 0 || i >= 128) return false;  // only after `over`
    return i < 64 ? ((lo >> i) & 1ull) : ((hi >> (i - 64)) & 1ull);
  }
  __host__ __device__ void push(int level, bool obj) {
    const int i = level - w0;
    if (i < 0 || i >= 128) {
      over = true;
      return;
    }
    if (i < 64) lo = obj ? (lo | (1ull << i)) : (lo & ~(1ull << i));
    else hi = obj ? (hi | (1ull << (i - 64))) : (hi & ~(1ull << (i - 64)));
  }
  __host__ __device__ void pop(int level) { floor_ = level < floor_ ? level : floor_; }
};

// A value starts with c (JM_TOP / JM_VALUE / JM_ARR_FIRST after whitespace):
// scan_once's dispatch.
template <class Stack>
__host__ __device__ void j_value_start(JState &st, Stack &stk, uint8_t c) {
  switch (c) {
    case '"':
      st.mode = JM_STR;
      st.key = 0;
      return;
    case '{':
    case '[':
      if (st.depth >= kJsonMaxDepth) {  // RecursionError
        st.decided = J_RAISE;
        return;
      }
      stk.push(st.depth, c == '{');
      ++st.depth;
      st.mode = c == '{' ? JM_OBJ_FIRST : JM_ARR_FIRST;
      return;
    case 'n': st.mode = JM_LIT; st.sub = 0; st.aux = 1; return;
    case 't': st.mode = JM_LIT; st.sub = 1; st.aux = 1; return;
    case 'f': st.mode = JM_LIT; st.sub = 2; st.aux = 1; return;
    case 'N': st.mode = JM_LIT; st.sub = 3; st.aux = 1; return;
    case 'I': st.mode = JM_LIT; st.sub = 4; st.aux = 1; return;
    case '-': st.mode = JM_NUM; st.sub = NP_MINUS; st.ndig = 0; st.isfloat = 0; return;
    default:
      if (j_digit(c)) {
        st.mode = JM_NUM;
        st.sub = c == '0' ? NP_ZERO : NP_INT;
        st.ndig = 1;
        st.isfloat = 0;
        return;
      }
      st.decided = J_TRUE;  // "Expecting value"
  }
}

// c after a value (JM_AFTER).
template <class Stack>
__host__ __device__ void j_after(JState &st, Stack &stk, uint8_t c) {
  if (j_ws(c)) return;
  if (st.depth == 0) {
    st.decided = J_FALSE;  // "Extra data"
    return;
  }
  const bool obj = stk.is_obj(st.depth - 1);
  if (c == (obj ? '}' : ']')) {
    stk.pop(--st.depth);
    return;  // still JM_AFTER
  }
  if (c == ',') {
    st.mode = obj ? JM_OBJ_KEY : JM_VALUE;
    return;
  }
  st.decided = J_TRUE;  // "Expecting ',' delimiter"
}

// The number ended before its last characters; ch is the first character
// after it.
template <class Stack>
__host__ __device__ void j_number_end(JState &st, Stack &stk, uint8_t ch) {
  if (!st.isfloat && st.ndig > kJsonIntDigits) {  // int() conversion limit
    st.decided = J_RAISE;
    return;
  }
  st.mode = JM_AFTER;
  j_after(st, stk, ch);
}

// One byte of the text.
template <class Stack>
__host__ __device__ void j_step(JState &st, Stack &stk, uint8_t c) {
  if (st.decided) return;
  if (st.first == 0) {  // the raw first character: '{' accepts any text
    st.first = 1;        // only "has the text begun" matters after it
    if (c == '{') {
      st.decided = J_TRUE;
      return;
    }
  }
  for (int replay = 0; replay < 2; ++replay) {  // at most one re-dispatch of c
    switch (st.mode) {
      case JM_TOP:
      case JM_VALUE:
        if (!j_ws(c)) j_value_start(st, stk, c);
        return;
      case JM_ARR_FIRST:
        if (j_ws(c)) return;
        if (c == ']') {
          stk.pop(--st.depth);
          st.mode = JM_AFTER;
          return;
        }
        j_value_start(st, stk, c);
        return;
      case JM_OBJ_FIRST:
      case JM_OBJ_KEY:
        if (j_ws(c)) return;
        if (st.mode == JM_OBJ_FIRST && c == '}') {
          stk.pop(--st.depth);
          st.mode = JM_AFTER;
          return;
        }
        if (c == '"') {
          st.mode = JM_STR;
          st.key = 1;
          return;
        }
        st.decided = J_TRUE;  // "Expecting property name enclosed in double quotes"
        return;
      case JM_AFTER_KEY:
        if (j_ws(c)) return;
        if (c == ':') {
          st.mode = JM_VALUE;
          return;
        }
        st.decided = J_TRUE;  // "Expecting ':' delimiter"
        return;
      case JM_AFTER:
        j_after(st, stk, c);
        return;
      case JM_STR:
        if (c == '"') {
          st.mode = st.key ? JM_AFTER_KEY : JM_AFTER;
        } else if (c == '\\') {
          st.mode = JM_ESC;
        } else if (c <= 0x1F) {
          st.decided = J_FALSE;  // "Invalid control character at"
        }
        return;
      case JM_ESC:
        if (c == 'u') {
          st.mode = JM_UHEX;
          st.aux = 0;
        } else if (c == '"' || c == '\\' || c == '/' || c == 'b' || c == 'f' || c == 'n' || c == 'r' ||
                   c == 't') {
          st.mode = JM_STR;
        } else {
          st.decided = J_FALSE;  // "Invalid \\escape"
        }
        return;
      case JM_UHEX:
        if (!j_hex(c)) {
          st.decided = J_FALSE;  // "Invalid \\uXXXX escape"
          return;
        }
        if (++st.aux == 4) st.mode = JM_UDONE;
        return;
      case JM_UDONE:  // a character follows the four digits: back in the string
        st.mode = JM_STR;
        continue;
      case JM_LIT: {
        if ((char)c != j_lit_char(st.sub, st.aux)) {
          st.decided = J_TRUE;  // the literal is not there: "Expecting value"
          return;
        }
        if (++st.aux == j_lit_len(st.sub)) st.mode = JM_AFTER;
        return;
      }
      case JM_NUM:
        switch (st.sub) {
          case NP_MINUS:
            if (c == 'I') {  // "-Infinity"
              st.mode = JM_LIT;
              st.sub = 5;
              st.aux = 2;
            } else if (j_digit(c)) {
              st.sub = c == '0' ? NP_ZERO : NP_INT;
              st.ndig = 1;
            } else {
              st.decided = J_TRUE;  // "-" alone: "Expecting value"
            }
            return;
          case NP_ZERO:
          case NP_INT:
            if (st.sub == NP_INT && j_digit(c)) {
              if (st.ndig <= kJsonIntDigits) ++st.ndig;
              return;
            }
            if (c == '.') {
              st.sub = NP_DOT;
              return;
            }
            if (c == 'e' || c == 'E') {
              st.sub = NP_E;
              return;
            }
            j_number_end(st, stk, c);
            return;
          case NP_DOT:
            if (j_digit(c)) {
              st.sub = NP_FRAC;
              st.isfloat = 1;
            } else {
              j_number_end(st, stk, '.');  // the '.' is not part of the number
            }
            return;
          case NP_FRAC:
            if (j_digit(c)) return;
            if (c == 'e' || c == 'E') {
              st.sub = NP_E;
              return;
            }
            j_number_end(st, stk, c);
            return;
          case NP_E:
            if (j_digit(c)) {
              st.sub = NP_EXP;
              st.isfloat = 1;
            } else if (c == '+' || c == '-') {
              st.sub = NP_ESIGN;
            } else {
              j_number_end(st, stk, 'e');  // no exponent: the 'e' follows the number
            }
            return;
          case NP_ESIGN:
            if (j_digit(c)) {
              st.sub = NP_EXP;
              st.isfloat = 1;
            } else {
              j_number_end(st, stk, 'e');
            }
            return;
          default:  // NP_EXP
            if (j_digit(c)) return;
            j_number_end(st, stk, c);
            return;
        }
      default:
        return;
    }
  }
}

// The class of the text read so far, at its end.
template <class Stack>
__host__ __device__ uint8_t j_finish(JState st, Stack &stk) {
  if (st.decided) return st.decided;
  if (st.first == 0) return J_TRUE;  // empty text
  switch (st.mode) {
    case JM_UHEX:
    case JM_UDONE:
      return J_FALSE;  // "Invalid \\uXXXX escape": the digits and one more character needed
    case JM_NUM:
      if (st.sub == NP_MINUS) return J_TRUE;
      if (!st.isfloat && st.ndig > kJsonIntDigits) return J_RAISE;
      if (st.sub == NP_DOT || st.sub == NP_E || st.sub == NP_ESIGN)  // a '.' or 'e' after the number
        return st.depth == 0 ? J_FALSE : J_TRUE;
      return J_TRUE;
    default:
      return J_TRUE;  // complete, or an "Expecting ..." / "Unterminated ..." at the end
  }
}

// ------------------------------------------------------------------ kernels
struct JsonVocab {
  const uint8_t *bytes;
  const int64_t *off;  // [V + 1]
  int64_t V;
  // optional fixed-width copy (ms_json_pack_vocab): token t's first 16 bytes
  // in packed[t], its length in lens[t] (kJsonLongToken when longer)
  const uint4 *packed;
  const uint8_t *lens;
  // optional order of the fixed-width copy (ms_json_pack_vocab_ordered):
  // packed[p] holds token order[p]; the mask kernel sets the bit of token
  // order[p] with an atomic OR into a row the dedup kernel zeroed
  const int32_t *order;
};

constexpr uint8_t kJsonLongToken = 255;
constexpr uint8_t kJsonPlain = 0x40;      // lens flag: no '"', '\\' or control byte (a short token)
constexpr uint8_t kJsonPlainTail = 0x20;  // lens flag: the same for every byte after the first
constexpr uint8_t kJsonLenMask = 0x1F;
constexpr uint8_t kJsonFirstStr = 4;      // first_dec: undecided, inside a string after the byte

// One thread per position p: token t = order[p] (t = p without an order) --
// its bytes zero-padded to 16 in packed[p], its length in lens[p] (with
// kJsonPlain when none of its bytes is '"', '\\' or below 0x20: such a token
// leaves a string body a string body; kJsonPlainTail when that holds for its
// bytes after the first).  An order entry outside [0, V) packs an empty token.
__global__ void ms_json_pack_kernel(const uint8_t *bytes, const int64_t *off, int64_t V, const int32_t *order,
                                    uint4 *packed, uint8_t *lens) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= V) return;
  const int64_t t = order ? (int64_t)order[p] : p;
  const bool in = t >= 0 && t < V;
  const int64_t b = in ? off[t] : 0, e = in ? off[t + 1] : 0;
  const int64_t n = e - b;
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  const int m = n < 16 ? (int)n : 16;
  bool plain = true, tail = true;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i < m) {
      const uint8_t c = bytes[b + i];
      w[i >> 2] |= (uint32_t)c << (8 * (i & 3));
      const bool pc = c >= 0x20 && c != '"' && c != '\\';
      plain = plain && pc;
      if (i > 0) tail = tail && pc;
    }
  }
  packed[p] = make_uint4(w[0], w[1], w[2], w[3]);
  lens[p] = n <= 16 ? (uint8_t)(n | (plain && n > 0 ? kJsonPlain : 0) | (tail && n > 0 ? kJsonPlainTail : 0))
                    : kJsonLongToken;
}

__device__ __forceinline__ void j_load_state(const uint32_t *g, uint32_t *sbits, JState &st) {
  const uint4 h = *reinterpret_cast<const uint4 *>(g);
  *reinterpret_cast<uint4 *>(&st) = h;
  const int words = (st.depth + 31) >> 5;
  for (int i = threadIdx.x; i < words; i += blockDim.x) sbits[i] = g[kJsonHeaderWords + i];
}

// One thread per row: the state after the row's prefix (ms_json_init) or after
// one more token (ms_json_advance).  The row's stack lives in global memory.

__global__ void ms_json_feed_kernel(uint32_t *states, int64_t B, const uint8_t *bytes, const int64_t *off,
                                    int64_t n_texts, const int64_t *which, int reset) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= B) return;
  uint32_t *g = states + row * kJsonStateWords;
  JState st;
  if (reset) {
    st = JState{J_UNDECIDED, JM_TOP, 0, 0, 0, 0, 0, 0, 0, 0};
  } else {
    *reinterpret_cast<uint4 *>(&st) = *reinterpret_cast<const uint4 *>(g);
  }
  JStackGlobal stk{g + kJsonHeaderWords};
  const int64_t t = which ? which[row] : row;  // the text appended to this row; < 0: none
  if (t >= 0 && t < n_texts) {
    for (int64_t i = off[t], e = off[t + 1]; i < e && !st.decided; ++i) j_step(st, stk, bytes[i]);
  }
  *reinterpret_cast<uint4 *>(g) = *reinterpret_cast<const uint4 *>(&st);
}

// grid (X, B): CTA (x, row) builds the mask words of its share of the
// vocabulary for `row`; lane l of a warp classifies token 32*w + l and a
// ballot packs the 32 answers into one word -- or, with an order, classifies
// the token at position 32*w + l and ORs its bit into the row.  row_status bits: 1 = some token makes
// the reference raise (its bit is 0), 2 = some token opens or closes more
// containers than JStackTok holds (its bit is 0).
// Rows in the same parse state get the same mask.  Row b's representative is
// the first row whose state is identical (header and the first `depth` stack
// bits); it is written as (rep + 1) << 8 into row_status[b], whose low byte
// collects the row's flags later.  Batches above kJsonDedupMax rows skip the
// search (every row its own representative).
constexpr int kJsonDedupMax = 1024;
__device__ __forceinline__ bool j_same_state(const uint32_t *x, const uint32_t *y) {
  // decided: every token gets the same answer, whatever the rest of the state
  const uint32_t dx = x[0] & 0xFFu;  // JState::decided
  if (dx != 0u && dx == (y[0] & 0xFFu)) return true;
  for (int i = 0; i < kJsonHeaderWords; ++i)
    if (x[i] != y[i]) return false;
  const int depth = (int)x[2];  // JState::depth
  const int words = depth >> 5, rem = depth & 31;
  for (int i = 0; i < words; ++i)
    if (x[kJsonHeaderWords + i] != y[kJsonHeaderWords + i]) return false;
  return rem == 0 || ((x[kJsonHeaderWords + words] ^ y[kJsonHeaderWords + words]) & ((1u << rem) - 1u)) == 0u;
}
// One warp per row b: lanes compare b's state with rows c < b, 32 at a time,
// the first match is b's representative.  With `zero` (ordered vocabulary) a
// representative's warp also clears its nwords mask words for the mask
// kernel's atomic ORs.
__global__ void ms_json_dedup_kernel(const uint32_t *states, int64_t B, int32_t *row_status, uint32_t *zero,
                                     int64_t mask_ld, int64_t nwords) {
  const int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= B) return;  // warp-uniform
  int64_t rep = b;
  if (B <= kJsonDedupMax) {
    const uint32_t *x = states + b * kJsonStateWords;
    for (int64_t c0 = 0; c0 < b; c0 += 32) {
      const int64_t c = c0 + lane;
      const bool same = c < b && j_same_state(x, states + c * kJsonStateWords);
      const uint32_t hit = __ballot_sync(0xFFFFFFFFu, same);
      if (hit) {
        rep = c0 + __ffs(hit) - 1;
        break;
      }
    }
  }
  if (lane == 0) row_status[b] = (int32_t)((rep + 1) << 8);
  if (zero && rep == b) {
    for (int64_t i = lane; i < nwords; i += 32) zero[b * mask_ld + i] = 0u;
  }
}

// Rows that share a representative take its mask; every row's status keeps
// only its flags.  One CTA per row.
__global__ void ms_json_mask_copy_kernel(uint32_t *mask, int64_t mask_ld, int64_t nwords, int32_t *row_status) {
  const int64_t row = blockIdx.x;
  const int32_t v = row_status[row];
  const int64_t rep = (int64_t)(v >> 8) - 1;
  if (rep != row) {
    const uint32_t *src = mask + rep * mask_ld;
    uint32_t *dst = mask + row * mask_ld;
    for (int64_t i0 = threadIdx.x; i0 < nwords; i0 += 8 * (int64_t)blockDim.x) {  // 8 loads in flight
      uint32_t q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t i = i0 + j * (int64_t)blockDim.x;
        q[j] = i < nwords ? src[i] : 0u;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t i = i0 + j * (int64_t)blockDim.x;
        if (i < nwords) dst[i] = q[j];
      }
    }
  }
  // the representative's low byte (its flags) is final; this kernel only
  // clears high bytes
  if (threadIdx.x == 0) row_status[row] = (rep != row ? row_status[rep] : v) & 0xFF;
}

__global__ void __launch_bounds__(kJsonThreads) ms_json_mask_kernel(const uint32_t *states, JsonVocab voc,
                                                                    uint32_t *mask, int64_t mask_ld,
                                                                    int32_t *row_status) {
  __shared__ uint32_t sbits[kJsonStackWords];
  __shared__ uint8_t first_dec[256];  // the row's decision after byte c alone (0: none yet)
  __shared__ int flags;
  const int row = blockIdx.y;
  // a row in the same state as an earlier row: ms_json_mask_copy_kernel fills it
  if ((row_status[row] >> 8) - 1 != row) return;
  const uint32_t *g = states + (int64_t)row * kJsonStateWords;
  JState st0;
  j_load_state(g, sbits, st0);
  if (threadIdx.x == 0) flags = 0;
  __syncthreads();
  const int64_t nwords = (voc.V + 31) >> 5;
  if (st0.decided) {  // every token gets the row's answer: whole words, token order
    const uint32_t fill = st0.decided == J_TRUE ? 0xFFFFFFFFu : 0u;
    for (int64_t w = (int64_t)blockIdx.x * kJsonThreads + threadIdx.x; w < nwords;
         w += (int64_t)gridDim.x * kJsonThreads) {
      const int tail = (int)(voc.V - w * 32);  // tokens in word w
      mask[(int64_t)row * mask_ld + w] = tail >= 32 ? fill : fill & ((1u << tail) - 1u);
    }
    if (st0.decided == J_RAISE && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(row_status + row, 1);
    return;
  }
  // a row inside a string body keeps it through a plain token (no '"', '\\'
  // or control byte), and a string body at the end of the text is "Unterminated
  // string": allowed (j_finish)
  const bool in_str = st0.mode == JM_STR;
  // a token whose first byte already decides takes that answer: once decided
  // the automaton ignores the rest of the text (j_step, j_finish)
  static_assert(kJsonThreads == 256, "one thread per first byte");
  {
    JState st = st0;
    JStackTok stk(sbits, st0.depth);
    j_step(st, stk, (uint8_t)threadIdx.x);
    // one byte never leaves the register window; a byte that opens (or keeps)
    // a string body is marked: a plain rest of the token keeps it open
    first_dec[threadIdx.x] = st.decided ? st.decided : (st.mode == JM_STR ? kJsonFirstStr : (uint8_t)J_UNDECIDED);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = (int64_t)gridDim.x * (kJsonThreads / 32);
  int my_flags = 0;
  for (int64_t w = (int64_t)blockIdx.x * (kJsonThreads / 32) + (threadIdx.x >> 5); w < nwords; w += warps_total) {
    const int64_t t = w * 32 + lane;
    // the token at position t (ordered vocabulary), or t itself; < 0: none
    int64_t tok = t < voc.V ? (voc.order ? (int64_t)voc.order[t] : t) : -1;
    if (tok >= voc.V) tok = -1;
    const int lb = tok >= 0 && voc.lens ? voc.lens[t] : kJsonLongToken;
    const int nb = lb == kJsonLongToken ? kJsonLongToken : (lb & kJsonLenMask);
    uint8_t r = J_FALSE;
    if (in_str && lb != kJsonLongToken && (lb & kJsonPlain)) {
      r = J_TRUE;  // the packed bytes are not needed
    } else {
      const uint4 q = tok >= 0 && voc.lens ? voc.packed[t] : make_uint4(0u, 0u, 0u, 0u);
      const uint8_t d = tok >= 0 && voc.lens && nb >= 1 ? first_dec[q.x & 0xFFu] : (uint8_t)J_UNDECIDED;
      if (d == kJsonFirstStr && lb != kJsonLongToken && (lb & kJsonPlainTail)) {
        r = J_TRUE;  // the first byte leaves a string body, the rest keeps it: "Unterminated string"
      } else if (d != J_UNDECIDED && d != kJsonFirstStr) {
        r = d;
        my_flags |= d == J_RAISE ? 1 : 0;
      } else if (tok >= 0) {
        JState st = st0;
        JStackTok stk(sbits, st0.depth);
        if (nb != kJsonLongToken) {  // the bytes from registers, low byte first
          uint64_t lo = (uint64_t)q.x | ((uint64_t)q.y << 32), hi = (uint64_t)q.z | ((uint64_t)q.w << 32);
          for (int i = 0; i < nb && !st.decided && !stk.over; ++i) {
            j_step(st, stk, (uint8_t)lo);
            lo = (lo >> 8) | (hi << 56);
            hi >>= 8;
          }
        } else {
          const int64_t b = voc.off[tok], e = voc.off[tok + 1];
          for (int64_t i = b; i < e && !st.decided && !stk.over; ++i) j_step(st, stk, voc.bytes[i]);
        }
        r = stk.over ? (uint8_t)J_UNDECIDED : j_finish(st, stk);
        my_flags |= r == J_RAISE ? 1 : (stk.over ? 2 : 0);
      }
    }
    if (voc.order) {
      if (r == J_TRUE) atomicOr(mask + (int64_t)row * mask_ld + (tok >> 5), 1u << (tok & 31));
    } else {
      const unsigned bits = __ballot_sync(0xFFFFFFFFu, r == J_TRUE);
      if (lane == 0) mask[(int64_t)row * mask_ld + w] = bits;
    }
  }
  if (my_flags) atomicOr(&flags, my_flags);
  __syncthreads();
  if (threadIdx.x == 0 && flags) atomicOr(row_status + row, flags);  // low byte: the flags
}

}  // namespace ms
