// LAMMPS ASCII dump reader and the synthetic dump writer of the trajectory
// example (examples/lammps_compress/src/main.rs:324-419), native like the
// reference's.
//
// Reader rules (same acceptance and error messages as the reference):
//   * lines are skipped until one whose trimmed text starts with
//     "ITEM: TIMESTEP"; the next line (the timestep) is not checked;
//   * then "ITEM: NUMBER OF ATOMS" (checked untrimmed), the atom count
//     (trimmed, unsigned decimal), "ITEM: BOX BOUNDS" plus three lines,
//     "ITEM: ATOMS <fields>" whose fields name the x, y and z columns;
//   * then one line per atom; the x/y/z tokens parse as f32, correctly
//     rounded, with Rust's float grammar (decimal or exponent forms, inf,
//     infinity, nan; no hex).
// The whole file is read once and scanned in place.
#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <system_error>
#include <string>
#include <string_view>

#include "nangila_host.hpp"

namespace ngl {
namespace host {
namespace {

struct Lines {
  const char* p;
  const char* end;
  // Next line including its '\n' (empty view at end of input).
  std::string_view next() {
    if (p >= end) return {};
    const char* nl = static_cast<const char*>(std::memchr(p, '\n', (size_t)(end - p)));
    const char* stop = nl ? nl + 1 : end;
    std::string_view s(p, (size_t)(stop - p));
    p = stop;
    return s;
  }
};

bool is_ws(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' || c == '\f'; }

std::string_view trim(std::string_view s) {
  size_t a = 0, b = s.size();
  while (a < b && is_ws(s[a])) ++a;
  while (b > a && is_ws(s[b - 1])) --b;
  return s.substr(a, b - a);
}

bool starts_with(std::string_view s, std::string_view pre) { return s.substr(0, pre.size()) == pre; }

// Whitespace-separated token i of s (empty view when there is none).
std::string_view token(std::string_view s, size_t want) {
  size_t i = 0, k = 0;
  while (true) {
    while (i < s.size() && is_ws(s[i])) ++i;
    if (i >= s.size()) return {};
    size_t j = i;
    while (j < s.size() && !is_ws(s[j])) ++j;
    if (k == want) return s.substr(i, j - i);
    ++k;
    i = j;
  }
}

bool ieq(std::string_view a, const char* b) {
  const size_t n = std::strlen(b);
  if (a.size() != n) return false;
  for (size_t i = 0; i < n; ++i)
    if ((a[i] | 0x20) != b[i]) return false;
  return true;
}

// f32 from a token with Rust's `str::parse::<f32>` grammar.
bool parse_f32(std::string_view t, float* out) {
  if (t.empty() || t.size() > 256) return false;
  std::string_view body = t;
  if (body[0] == '+' || body[0] == '-') body.remove_prefix(1);
  if (ieq(body, "inf") || ieq(body, "infinity") || ieq(body, "nan")) {
    const bool neg = t[0] == '-';
    *out = body[0] == 'n' || body[0] == 'N' ? NAN : (neg ? -INFINITY : INFINITY);
    return true;
  }
  // digits [. digits] [e [+-] digits], at least one mantissa digit
  size_t i = 0, mant = 0;
  while (i < body.size() && body[i] >= '0' && body[i] <= '9') ++i, ++mant;
  if (i < body.size() && body[i] == '.') {
    ++i;
    while (i < body.size() && body[i] >= '0' && body[i] <= '9') ++i, ++mant;
  }
  if (mant == 0) return false;
  if (i < body.size() && (body[i] == 'e' || body[i] == 'E')) {
    ++i;
    if (i < body.size() && (body[i] == '+' || body[i] == '-')) ++i;
    size_t ed = 0;
    while (i < body.size() && body[i] >= '0' && body[i] <= '9') ++i, ++ed;
    if (ed == 0) return false;
  }
  if (i != body.size()) return false;
  // from_chars is correctly rounded like Rust's parse; it takes no '+' and
  // reports overflow/underflow instead of rounding to inf or zero, so those
  // rare tokens go through strtof, which rounds them.
  const char* b0 = t.data() + (t[0] == '+' ? 1 : 0);
  const char* b1 = t.data() + t.size();
  float v = 0.0f;
  const auto r = std::from_chars(b0, b1, v, std::chars_format::general);
  if (r.ec == std::errc() && r.ptr == b1) {
    *out = v;
    return true;
  }
  char buf[260];
  std::memcpy(buf, t.data(), t.size());
  buf[t.size()] = '\0';
  char* endp = nullptr;
  v = std::strtof(buf, &endp);
  if (endp != buf + t.size()) return false;
  *out = v;
  return true;
}

bool parse_usize(std::string_view t, size_t* out) {
  if (!t.empty() && t[0] == '+') t.remove_prefix(1);
  if (t.empty()) return false;
  size_t v = 0;
  for (char c : t) {
    if (c < '0' || c > '9') return false;
    const size_t d = (size_t)(c - '0');
    if (v > (SIZE_MAX - d) / 10) return false;
    v = v * 10 + d;
  }
  *out = v;
  return true;
}

}  // namespace

std::vector<Floats> lammps_read_dump_text(const char* text, size_t size) {
  Lines in{text, text + size};
  std::vector<Floats> snaps;
  while (true) {
    std::string_view line = in.next();
    if (line.empty()) break;
    if (!starts_with(trim(line), "ITEM: TIMESTEP")) continue;
    in.next();  // timestep value
    line = in.next();
    if (!starts_with(line, "ITEM: NUMBER OF ATOMS"))
      throw std::runtime_error("unexpected format, expected NUMBER OF ATOMS line");
    size_t natoms = 0;
    if (!parse_usize(trim(in.next()), &natoms)) throw std::runtime_error("parse natoms");
    line = in.next();
    if (!starts_with(line, "ITEM: BOX BOUNDS")) throw std::runtime_error("unexpected format, expected BOX BOUNDS line");
    for (int i = 0; i < 3; ++i) in.next();
    line = in.next();
    if (!starts_with(line, "ITEM: ATOMS")) throw std::runtime_error("expected ATOMS header");
    long xi = -1, yi = -1, zi = -1;
    for (size_t f = 0;; ++f) {
      const std::string_view col = token(line, f + 2);  // fields follow "ITEM:" and "ATOMS"
      if (col.empty()) break;
      if (col == "x") xi = (long)f;
      if (col == "y") yi = (long)f;
      if (col == "z") zi = (long)f;
    }
    if (xi < 0) throw std::runtime_error("x column not found");
    if (yi < 0) throw std::runtime_error("y column not found");
    if (zi < 0) throw std::runtime_error("z column not found");
    // Each atom line holds at least one character, so a count above the
    // remaining bytes can only end at the EOF error; reserve no more.
    Floats snap;
    snap.reserve(3 * std::min(natoms, (size_t)(in.end - in.p)));
    for (size_t a = 0; a < natoms; ++a) {
      line = in.next();
      if (line.empty()) throw std::runtime_error("unexpected EOF reading atoms");
      const long idx[3] = {xi, yi, zi};
      static const char* const kMissing[3] = {"x missing", "y missing", "z missing"};
      static const char* const kParse[3] = {"x parse", "y parse", "z parse"};
      for (int c = 0; c < 3; ++c) {
        const std::string_view t = token(line, (size_t)idx[c]);
        if (t.empty()) throw std::runtime_error(kMissing[c]);
        float v;
        if (!parse_f32(t, &v)) throw std::runtime_error(kParse[c]);
        snap.push_back(v);
      }
    }
    snaps.push_back(std::move(snap));
  }
  return snaps;
}

std::vector<Floats> lammps_read_dump(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("open " + path);
  f.seekg(0, std::ios::end);
  const std::streamoff n = f.tellg();
  f.seekg(0, std::ios::beg);
  std::string text((size_t)(n > 0 ? n : 0), '\0');
  if (n > 0 && !f.read(&text[0], n)) throw std::runtime_error("read " + path);
  return lammps_read_dump_text(text.data(), text.size());
}

void lammps_write_dump(const std::string& path, size_t atoms, size_t steps) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw std::runtime_error("create " + path);
  std::vector<char> buf(1 << 20);
  std::setvbuf(f, buf.data(), _IOFBF, buf.size());
  for (size_t t = 0; t < steps; ++t) {
    std::fprintf(f, "ITEM: TIMESTEP\n%zu\nITEM: NUMBER OF ATOMS\n%zu\nITEM: BOX BOUNDS xx yy zz\n", t, atoms);
    std::fputs("0 10\n0 10\n0 10\nITEM: ATOMS id type x y z\n", f);
    const float tt = (float)t * 0.1f;
    for (size_t i = 0; i < atoms; ++i) {
      const float phase = tt + (float)i * 0.001f;
      const float x = std::cos(phase), y = std::sin(phase), z = std::cos(phase * 0.5f);
      std::fprintf(f, "%zu 1 %.6f %.6f %.6f\n", i + 1, (double)x, (double)y, (double)z);
    }
  }
  const bool bad = std::ferror(f) != 0;
  std::fclose(f);
  if (bad) throw std::runtime_error("write " + path);
}

}  // namespace host
}  // namespace ngl
