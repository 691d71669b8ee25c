// Checkpoint codec: CRC32 (IEEE 802.3), the reference's float text encoding, and streaming helpers
// for the binary containers. Host-only C++ (g++), exported with a C ABI for ctypes.
//
// Formats reproduced byte for byte (the layouts must match to read and write the reference's files):
//   * per-tensor v2 binary: magic "BRAIN   ", u32 version 2, endian/dtype/compression/reserved bytes,
//     u32 rank, u64 dims, u32 CRC32 of the payload, u64 payload length, payload as f64 LE
//     (crates/brain-core/src/serialization.rs:53-77, 190-330);
//   * TensorArchive "BRAIN_ARCHIVE\0" (serialization.rs:414-553) and the ".bn" BrainModelFile
//     "BRAIN_BN" with a trailing CRC32 over every preceding byte (serialization.rs:574-760);
//   * the BRAIN_STATE_V1 text checkpoint, whose values are Rust f64 Display strings: the shortest
//     digits that round-trip, written without an exponent ("0.0000001", "100000000000000000000"),
//     with "NaN", "inf", "-inf" and "-0" (crates/brain-train/src/lib.rs:938-1069).
// The binary layouts themselves are assembled in Python (brain_b200/checkpoint); this file holds the
// byte-level hot loops: CRC over gigabytes and float formatting/parsing over millions of values.
#include <charconv>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>

#define BRAIN_API extern "C" __attribute__((visibility("default")))

namespace {

// Slicing-by-8 tables for the reflected polynomial 0xEDB88320.
struct CrcTables {
  uint32_t t[8][256];
  CrcTables() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? (c >> 1) ^ 0xEDB88320u : (c >> 1);
      t[0][i] = c;
    }
    for (uint32_t i = 0; i < 256; ++i)
      for (int s = 1; s < 8; ++s) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xFF];
  }
};
const CrcTables& tables() {
  static CrcTables tb;
  return tb;
}

// Shortest round-trip digits of v (finite, non-zero), written as plain decimal like Rust's Display.
size_t format_one(double v, char* out) {
  if (std::isnan(v)) {
    std::memcpy(out, "NaN", 3);
    return 3;
  }
  if (std::isinf(v)) {
    if (v < 0) {
      std::memcpy(out, "-inf", 4);
      return 4;
    }
    std::memcpy(out, "inf", 3);
    return 3;
  }
  size_t n = 0;
  if (std::signbit(v)) {
    out[n++] = '-';
    v = -v;
  }
  if (v == 0.0) {
    out[n++] = '0';
    return n;
  }
  char sci[64];
  auto r = std::to_chars(sci, sci + sizeof(sci), v, std::chars_format::scientific);
  // sci = d[.ddd]e[+-]XX
  char digits[32];
  int nd = 0;
  const char* p = sci;
  while (p < r.ptr && *p != 'e') {
    if (*p != '.') digits[nd++] = *p;
    ++p;
  }
  // exponent: to_chars does not NUL-terminate, so parse only up to r.ptr
  const char* q = p + 1;
  if (q < r.ptr && *q == '+') ++q;
  int exp10 = 0;  // value = d.ddd * 10^exp10
  std::from_chars(q, r.ptr, exp10);
  const int point = exp10 + 1;     // digits before the decimal point
  if (point <= 0) {
    out[n++] = '0';
    out[n++] = '.';
    for (int i = 0; i < -point; ++i) out[n++] = '0';
    for (int i = 0; i < nd; ++i) out[n++] = digits[i];
  } else if (point >= nd) {
    for (int i = 0; i < nd; ++i) out[n++] = digits[i];
    for (int i = nd; i < point; ++i) out[n++] = '0';
  } else {
    for (int i = 0; i < point; ++i) out[n++] = digits[i];
    out[n++] = '.';
    for (int i = point; i < nd; ++i) out[n++] = digits[i];
  }
  return n;
}

}  // namespace

// Streaming CRC32: pass state = 0xFFFFFFFF initially, finalize with crc = state ^ 0xFFFFFFFF.
BRAIN_API uint32_t brain_crc32_update(uint32_t state, const uint8_t* data, int64_t n) {
  const auto& T = tables().t;
  int64_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint32_t lo, hi;
    std::memcpy(&lo, data + i, 4);
    std::memcpy(&hi, data + i + 4, 4);
    lo ^= state;
    state = T[7][lo & 0xFF] ^ T[6][(lo >> 8) & 0xFF] ^ T[5][(lo >> 16) & 0xFF] ^ T[4][lo >> 24] ^
            T[3][hi & 0xFF] ^ T[2][(hi >> 8) & 0xFF] ^ T[1][(hi >> 16) & 0xFF] ^ T[0][hi >> 24];
  }
  for (; i < n; ++i) state = (state >> 8) ^ T[0][(state ^ data[i]) & 0xFF];
  return state;
}

BRAIN_API uint32_t brain_crc32(const uint8_t* data, int64_t n) {
  return brain_crc32_update(0xFFFFFFFFu, data, n) ^ 0xFFFFFFFFu;
}

// Comma-joined Rust-Display strings of vals[0..n). Returns bytes written, or -(bytes needed) if cap
// is too small. A value needs at most 350 bytes (1e308 written out), so cap = 350*n is always enough.
BRAIN_API int64_t brain_format_f64(const double* vals, int64_t n, char* out, int64_t cap) {
  int64_t w = 0;
  char tmp[400];
  for (int64_t i = 0; i < n; ++i) {
    size_t k = format_one(vals[i], tmp);
    int64_t need = (int64_t)k + (i ? 1 : 0);
    if (w + need > cap) return -(w + need + 350 * (n - i));
    if (i) out[w++] = ',';
    std::memcpy(out + w, tmp, k);
    w += (int64_t)k;
  }
  return w;
}

// Parse a comma-separated list of decimal floats (Rust f64 syntax incl. NaN/inf/-inf/exponents).
// Returns the number of values, or -1 - index of the first bad token.
BRAIN_API int64_t brain_parse_f64(const char* s, int64_t len, double* out, int64_t max_out) {
  if (len == 0) return 0;
  int64_t count = 0, start = 0;
  std::string tok;
  for (int64_t i = 0; i <= len; ++i) {
    if (i == len || s[i] == ',') {
      if (count >= max_out) return -1 - count;
      tok.assign(s + start, s + i);
      double v;
      if (tok == "NaN") v = std::nan("");
      else if (tok == "inf" || tok == "+inf" || tok == "infinity" || tok == "+infinity") v = INFINITY;
      else if (tok == "-inf" || tok == "-infinity") v = -INFINITY;
      else {
        if (tok.empty()) return -1 - count;
        char* end = nullptr;
        v = std::strtod(tok.c_str(), &end);
        if (end != tok.c_str() + tok.size()) return -1 - count;
        // strtod accepts hex / "nan(...)" forms Rust rejects
        for (char c : tok)
          if (!((c >= '0' && c <= '9') || c == '.' || c == 'e' || c == 'E' || c == '+' || c == '-'))
            return -1 - count;
      }
      out[count++] = v;
      start = i + 1;
    }
  }
  return count;
}

// ---------------------------------------------------------------------------------------------
// Reference RNG streams for oracle parity with the CPU framework (crates/brain-core/src/random.rs):
// SplitMix64 (random.rs:118-124), BrainRng = xorshift128+ seeded by SplitMix64(seed + 1)
// (random.rs:194-234), next_f64 = (u64 >> 11) * 2^-53, and Tensor::randn's Box-Muller cosine branch
// with u1 = max(1 - next_f64, 1e-15) (crates/brain-core/src/tensor/impl.rs:222-236).
// The state (two u64) is updated in place so streams continue across calls.
// ---------------------------------------------------------------------------------------------
namespace {
inline uint64_t splitmix_next(uint64_t& s) {
  s += 0x9E3779B97F4A7C15ull;
  uint64_t z = s;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
inline uint64_t xorshift_next(uint64_t* st) {
  uint64_t s1 = st[0];
  const uint64_t s0 = st[1];
  const uint64_t result = s0 + s1;
  st[0] = s0;
  s1 ^= s1 << 23;
  st[1] = s1 ^ s0 ^ (s1 >> 17) ^ (s0 >> 26);
  return result;
}
inline double next_f64(uint64_t* st) { return (double)(xorshift_next(st) >> 11) * (1.0 / 9007199254740992.0); }
}  // namespace

BRAIN_API void brain_rng_seed(uint64_t seed, uint64_t* state_out) {
  uint64_t sm = seed + 1;
  state_out[0] = splitmix_next(sm);
  state_out[1] = splitmix_next(sm);
  if (state_out[0] == 0 && state_out[1] == 0) {
    state_out[0] = 0xDEADBEEFCAFEBABEull;
    state_out[1] = 0x123456789ABCDEF0ull;
  }
}

// mode 0: uniform [0,1) doubles; 1: standard normal (Box-Muller cosine branch); 2: raw u64 as doubles
BRAIN_API void brain_rng_fill(uint64_t* state, int64_t n, double* out, int mode) {
  for (int64_t i = 0; i < n; ++i) {
    if (mode == 0) {
      out[i] = next_f64(state);
    } else if (mode == 1) {
      double u1 = 1.0 - next_f64(state);
      if (u1 < 1e-15) u1 = 1e-15;
      const double u2 = next_f64(state);
      out[i] = std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * 3.14159265358979323846 * u2);
    } else {
      out[i] = (double)xorshift_next(state);
    }
  }
}
