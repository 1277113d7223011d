// Minimal HDF5 writer and reader; see hdf5_io.hpp for the supported subset.
// Every structure below follows the HDF5 File Format Specification
// (superblock, object headers and their messages, version-1 B-trees, symbol
// table nodes, local and global heaps).  Little-endian, 8-byte offsets and
// lengths on write; the reader takes the sizes from the superblock.
#include "hdf5_io.hpp"

#include <algorithm>
#include <cstring>
#include <set>

namespace ngl {
namespace h5 {
namespace {

constexpr uint64_t kUndef = ~uint64_t(0);
const char kSignature[8] = {'\x89', 'H', 'D', 'F', '\r', '\n', '\x1a', '\n'};
// Group B-tree "K" values written to the superblock.  A reader sizes every
// symbol table node for 2 * leaf K entries and every group B-tree node for
// 2 * internal K children, so nodes are written at those full sizes.
constexpr int kLeafK = 4;
constexpr int kInternalK = 16;
constexpr uint64_t kEntryBytes = 40;  // symbol table entry with 8-byte offsets
constexpr uint64_t kSnodBytes = 8 + 2 * kLeafK * kEntryBytes;
constexpr uint64_t kTreeBytes = 24 + 2 * kInternalK * 8 + (2 * kInternalK + 1) * 8;
// Local heap free-list value meaning "no free block" (what libhdf5 writes
// and expects; the undefined address is rejected by it as a bad free list).
constexpr uint64_t kHeapNoFree = 1;

enum : uint16_t {
  kMsgNil = 0x0000,
  kMsgDataspace = 0x0001,
  kMsgLinkInfo = 0x0002,
  kMsgDatatype = 0x0003,
  kMsgFill = 0x0005,
  kMsgLink = 0x0006,
  kMsgLayout = 0x0008,
  kMsgAttribute = 0x000C,
  kMsgContinuation = 0x0010,
  kMsgSymbolTable = 0x0011,
};

uint64_t elements(const std::vector<uint64_t>& shape) {
  uint64_t n = 1;
  for (uint64_t d : shape) n *= d;
  return n;
}

// Byte count of n elements of esz bytes; corrupt sizes (past 2^48 bytes, or
// overflowing) are rejected before anything is allocated from them.
uint64_t checked_bytes(const std::vector<uint64_t>& shape, uint64_t esz) {
  constexpr uint64_t kLimit = uint64_t(1) << 48;
  uint64_t n = esz;
  for (uint64_t d : shape) {
    if (d != 0 && n > kLimit / d) throw Error("dataspace too large (corrupt file?)");
    n *= d;
  }
  if (n > kLimit) throw Error("dataspace too large (corrupt file?)");
  return n;
}

void check_value(const Value& v, const std::string& what) {
  const bool ok_kind = (v.kind == 'u' || v.kind == 'i') ? (v.size == 1 || v.size == 2 || v.size == 4 || v.size == 8)
                       : v.kind == 'f'                  ? (v.size == 4 || v.size == 8)
                       : v.kind == 'S'                  ? v.size >= 1
                                                        : false;
  if (!ok_kind) throw Error(what + ": unsupported element type");
  if (elements(v.shape) * (uint64_t)v.size != v.bytes.size())
    throw Error(what + ": data size does not match its shape and element size");
}

// ------------------------------------------------------------------ writer
struct Buf {
  std::string b;
  uint64_t pos() const { return b.size(); }
  void align8() { b.resize((b.size() + 7) & ~size_t(7), '\0'); }
  void le(uint64_t v, int n) {
    for (int i = 0; i < n; ++i) b.push_back((char)((v >> (8 * i)) & 0xff));
  }
  void u8(uint64_t v) { le(v, 1); }
  void u16(uint64_t v) { le(v, 2); }
  void u32(uint64_t v) { le(v, 4); }
  void u64(uint64_t v) { le(v, 8); }
  void raw(const std::string& s) { b += s; }
  void zeros(size_t n) { b.append(n, '\0'); }
  void pad_to(uint64_t start, uint64_t bytes) { b.resize(start + bytes, '\0'); }
};

std::string pad8(std::string s) {
  s.resize((s.size() + 7) & ~size_t(7), '\0');
  return s;
}

// Datatype message body: fixed-point (class 0), IEEE float (class 1) or a
// null-padded ASCII fixed-length string (class 3), version 1.
std::string datatype_body(const Value& v) {
  Buf o;
  if (v.kind == 'u' || v.kind == 'i') {
    o.u8(0x10);                          // version 1, class 0
    o.u8(v.kind == 'i' ? 0x08 : 0x00);   // little endian, zero padding, signedness
    o.u8(0);
    o.u8(0);
    o.u32(v.size);
    o.u16(0);                            // bit offset
    o.u16(8 * v.size);                   // bit precision
  } else if (v.kind == 'f') {
    const bool dbl = v.size == 8;
    o.u8(0x11);                          // version 1, class 1
    o.u8(0x20);                          // little endian, implied leading mantissa bit
    o.u8(dbl ? 63 : 31);                 // sign bit position
    o.u8(0);
    o.u32(v.size);
    o.u16(0);                            // bit offset
    o.u16(8 * v.size);                   // bit precision
    o.u8(dbl ? 52 : 23);                 // exponent location
    o.u8(dbl ? 11 : 8);                  // exponent size
    o.u8(0);                             // mantissa location
    o.u8(dbl ? 52 : 23);                 // mantissa size
    o.u32(dbl ? 1023 : 127);             // exponent bias
  } else {
    o.u8(0x13);                          // version 1, class 3
    o.u8(0x01);                          // null padded, ASCII
    o.u8(0);
    o.u8(0);
    o.u32(v.size);
  }
  return o.b;
}

// Dataspace message version 1 (rank 0 = scalar).
std::string dataspace_body(const std::vector<uint64_t>& shape) {
  Buf o;
  o.u8(1);
  o.u8(shape.size());
  o.u8(0);  // no maximum dimensions
  o.u8(0);
  o.u32(0);
  for (uint64_t d : shape) o.u64(d);
  return o.b;
}

// Attribute message version 1: name, datatype and dataspace each padded to
// 8 bytes, then the raw value.
std::string attribute_body(const Attr& a) {
  check_value(a.value, "attribute " + a.name);
  const std::string name = a.name + '\0';
  const std::string dt = datatype_body(a.value), ds = dataspace_body(a.value.shape);
  Buf o;
  o.u8(1);
  o.u8(0);
  o.u16(name.size());
  o.u16(dt.size());
  o.u16(ds.size());
  o.raw(pad8(name));
  o.raw(pad8(dt));
  o.raw(pad8(ds));
  o.raw(a.value.bytes);
  return o.b;
}

using Msgs = std::vector<std::pair<uint16_t, std::string>>;

// Version-1 object header: 16-byte prefix, then 8-byte aligned messages.
uint64_t write_object_header(Buf& f, const Msgs& msgs) {
  f.align8();
  const uint64_t at = f.pos();
  uint64_t size = 0;
  for (const auto& m : msgs) {
    const uint64_t body = pad8(m.second).size();
    if (body > 0xffff) throw Error("object header message larger than 64 KiB");
    size += 8 + body;
  }
  f.u8(1);              // version
  f.u8(0);
  f.u16(msgs.size());   // number of messages
  f.u32(1);             // reference count
  f.u32(size);          // header data size
  f.u32(0);             // alignment padding
  for (const auto& m : msgs) {
    const std::string body = pad8(m.second);
    f.u16(m.first);
    f.u16(body.size());
    f.u8(0);  // flags
    f.zeros(3);
    f.raw(body);
  }
  return at;
}

uint64_t write_dataset(Buf& f, const Object& d) {
  check_value(d.data, "dataset " + d.name);
  uint64_t data_at = kUndef;
  if (!d.data.bytes.empty()) {
    f.align8();
    data_at = f.pos();
    f.raw(d.data.bytes);
  }
  Msgs msgs;
  msgs.push_back({kMsgDataspace, dataspace_body(d.data.shape)});
  msgs.push_back({kMsgDatatype, datatype_body(d.data)});
  {
    Buf fill;  // fill value message version 2: allocated late, written if set, undefined
    fill.u8(2);
    fill.u8(2);
    fill.u8(2);
    fill.u8(0);
    msgs.push_back({kMsgFill, fill.b});
  }
  {
    Buf lay;  // layout message version 3, contiguous storage
    lay.u8(3);
    lay.u8(1);
    lay.u64(data_at);
    lay.u64(d.data.bytes.size());
    msgs.push_back({kMsgLayout, lay.b});
  }
  for (const auto& a : d.attrs) msgs.push_back({kMsgAttribute, attribute_body(a)});
  return write_object_header(f, msgs);
}

struct GroupAt {
  uint64_t header, btree, heap;
};

GroupAt write_group(Buf& f, const std::vector<Object>& objs, const std::vector<std::vector<int>>& kids, int gi,
                    int depth) {
  if (depth > 64) throw Error("group nesting deeper than 64 levels");
  struct Entry {
    std::string name;
    uint64_t header;
    bool group;
    uint64_t btree, heap;
    uint64_t name_off;
  };
  std::vector<int> order = kids[gi];
  std::sort(order.begin(), order.end(), [&](int a, int b) { return objs[a].name < objs[b].name; });
  std::vector<Entry> entries;
  for (size_t i = 0; i < order.size(); ++i) {
    const Object& o = objs[order[i]];
    if (o.name.empty() || o.name.find('/') != std::string::npos || o.name.find('\0') != std::string::npos)
      throw Error("invalid link name '" + o.name + "'");
    if (i > 0 && objs[order[i - 1]].name == o.name) throw Error("duplicate link name '" + o.name + "'");
    if (o.is_group) {
      const GroupAt g = write_group(f, objs, kids, order[i], depth + 1);
      entries.push_back({o.name, g.header, true, g.btree, g.heap, 0});
    } else {
      entries.push_back({o.name, write_dataset(f, o), false, 0, 0, 0});
    }
  }
  if (entries.size() > (size_t)(2 * kLeafK) * (2 * kInternalK))
    throw Error("more than 256 links in one group");
  // Local heap: the empty name at offset 0, then every link name,
  // null-terminated and padded to 8 bytes.
  Buf names;
  names.zeros(8);
  for (auto& e : entries) {
    e.name_off = names.pos();
    names.raw(e.name);
    names.u8(0);
    names.align8();
  }
  f.align8();
  const uint64_t heap = f.pos();
  f.raw("HEAP");
  f.u8(0);
  f.zeros(3);
  f.u64(names.pos());   // data segment size
  f.u64(kHeapNoFree);   // free list: none
  f.u64(heap + 32);     // data segment follows the header
  f.raw(names.b);
  // Symbol table nodes of up to 2 * leaf K entries, sorted by name.
  std::vector<uint64_t> snods, last_name;
  for (size_t s = 0; s < entries.size(); s += 2 * kLeafK) {
    const size_t e = std::min(entries.size(), s + 2 * kLeafK);
    f.align8();
    const uint64_t at = f.pos();
    f.raw("SNOD");
    f.u8(1);
    f.u8(0);
    f.u16(e - s);
    for (size_t i = s; i < e; ++i) {
      const Entry& x = entries[i];
      f.u64(x.name_off);
      f.u64(x.header);
      f.u32(x.group ? 1 : 0);  // cache type 1: the scratch pad holds the group's B-tree and heap
      f.u32(0);
      f.u64(x.group ? x.btree : 0);
      f.u64(x.group ? x.heap : 0);
    }
    f.pad_to(at, kSnodBytes);
    snods.push_back(at);
    last_name.push_back(entries[e - 1].name_off);
  }
  // One leaf node of the group B-tree: key 0 is the empty name, key i+1 the
  // last (greatest) name of child i.
  f.align8();
  const uint64_t btree = f.pos();
  f.raw("TREE");
  f.u8(0);  // group node
  f.u8(0);  // leaf level
  f.u16(snods.size());
  f.u64(kUndef);  // left sibling
  f.u64(kUndef);  // right sibling
  f.u64(0);
  for (size_t i = 0; i < snods.size(); ++i) {
    f.u64(snods[i]);
    f.u64(last_name[i]);
  }
  f.pad_to(btree, kTreeBytes);
  Buf st;
  st.u64(btree);
  st.u64(heap);
  Msgs msgs{{kMsgSymbolTable, st.b}};
  for (const auto& a : objs[gi].attrs) msgs.push_back({kMsgAttribute, attribute_body(a)});
  return {write_object_header(f, msgs), btree, heap};
}

// ------------------------------------------------------------------ reader
struct Reader {
  const std::string& f;
  uint64_t base = 0;
  int so = 8, sl = 8;  // sizes of offsets and lengths

  explicit Reader(const std::string& file) : f(file) {}

  void need(uint64_t at, uint64_t n) const {
    if (at > f.size() || n > f.size() - at) throw Error("truncated or corrupt HDF5 file");
  }
  uint64_t le(uint64_t at, int n) const {
    need(at, n);
    uint64_t v = 0;
    for (int i = 0; i < n; ++i) v |= (uint64_t)(uint8_t)f[at + i] << (8 * i);
    return v;
  }
  uint64_t off(uint64_t at) const {
    const uint64_t v = le(at, so);
    return (so < 8 && v == ((uint64_t(1) << (8 * so)) - 1)) ? kUndef : v;
  }
  uint64_t len(uint64_t at) const { return le(at, sl); }
  uint64_t abs(uint64_t rel) const {
    if (rel == kUndef) throw Error("undefined address where an object was expected");
    return base + rel;
  }
  bool sig(uint64_t at, const char* s) const {
    need(at, 4);
    return std::memcmp(f.data() + at, s, 4) == 0;
  }
  std::string cstr(uint64_t at) const {
    need(at, 1);
    const char* p = f.data() + at;
    const size_t n = strnlen(p, f.size() - at);
    if (at + n >= f.size()) throw Error("unterminated name");
    return std::string(p, n);
  }
};

struct Msg {
  uint16_t type;
  uint64_t at;  // absolute position of the message body
  uint64_t size;
};

// Messages of the object header at absolute position `at`, following
// continuation blocks.
std::vector<Msg> object_messages(const Reader& r, uint64_t at) {
  std::vector<Msg> out;
  std::vector<std::pair<uint64_t, uint64_t>> blocks;  // (start, end) of message areas
  bool v2 = false;
  int v2_flags = 0;
  if (r.sig(at, "OHDR")) {
    v2 = true;
    r.need(at, 6);
    if ((uint8_t)r.f[at + 4] != 2) throw Error("unsupported object header version");
    v2_flags = (uint8_t)r.f[at + 5];
    uint64_t q = at + 6;
    if (v2_flags & 0x20) q += 16;
    if (v2_flags & 0x10) q += 4;
    const int nb = 1 << (v2_flags & 3);
    const uint64_t size = r.le(q, nb);
    q += nb;
    blocks.push_back({q, q + size});
  } else {
    r.need(at, 16);
    if ((uint8_t)r.f[at] != 1) throw Error("unsupported object header version");
    const uint64_t size = r.le(at + 8, 4);
    blocks.push_back({at + 16, at + 16 + size});
  }
  std::set<uint64_t> seen;
  for (size_t bi = 0; bi < blocks.size(); ++bi) {
    uint64_t p = blocks[bi].first;
    const uint64_t end = blocks[bi].second;
    r.need(p, end - p);
    const uint64_t hdr = v2 ? (4 + ((v2_flags & 0x04) ? 2 : 0)) : 8;
    while (p + hdr <= end) {
      uint16_t type;
      uint64_t size;
      if (v2) {
        type = (uint8_t)r.f[p];
        size = r.le(p + 1, 2);
      } else {
        type = (uint16_t)r.le(p, 2);
        size = r.le(p + 2, 2);
      }
      const uint64_t body = p + hdr;
      if (body + size > end) throw Error("object header message runs past its block");
      out.push_back({type, body, size});
      if (type == kMsgContinuation) {
        const uint64_t ca = r.abs(r.off(body)), cl = r.len(body + r.so);
        if (cl > 0 && seen.insert(ca).second) {
          if (v2) {
            if (!r.sig(ca, "OCHK")) throw Error("bad object header continuation block");
            if (cl < 8) throw Error("bad object header continuation length");
            blocks.push_back({ca + 4, ca + cl - 4});
          } else {
            blocks.push_back({ca, ca + cl});
          }
        }
      }
      p = body + size;
    }
    if (blocks.size() > 4096) throw Error("too many object header continuation blocks");
  }
  return out;
}

struct Type {
  int cls = -1;
  char kind = 'V';
  int size = 0;
  bool big_endian = false;
  bool vlen_string = false;
};

Type parse_type(const Reader& r, uint64_t at, uint64_t size) {
  if (size < 8) throw Error("short datatype message");
  r.need(at, 8);
  Type t;
  const uint8_t b0 = r.f[at], b1 = r.f[at + 1];
  t.cls = b0 & 0x0f;
  t.size = (int)r.le(at + 4, 4);
  switch (t.cls) {
    case 0:
      t.kind = (b1 & 0x08) ? 'i' : 'u';
      t.big_endian = b1 & 0x01;
      break;
    case 1:
      t.kind = 'f';
      t.big_endian = b1 & 0x01;
      if (b1 & 0x40) throw Error("VAX-ordered floats are not supported");
      break;
    case 3:
      t.kind = 'S';
      break;
    case 9:
      if ((b1 & 0x0f) != 1) throw Error("variable-length sequences are not supported");
      t.kind = 'S';
      t.vlen_string = true;
      break;
    default:
      t.kind = 'V';  // kept as opaque bytes
  }
  bool ok;
  if (t.vlen_string) ok = true;  // elements are heap references of a fixed size
  else if (t.kind == 'u' || t.kind == 'i') ok = t.size == 1 || t.size == 2 || t.size == 4 || t.size == 8;
  else if (t.kind == 'f') ok = t.size == 2 || t.size == 4 || t.size == 8;
  else ok = t.size >= 1 && t.size <= (1 << 20);
  if (!ok) throw Error("unsupported or corrupt datatype size");
  return t;
}

// Dataspace: shape (empty for scalar); false for a null dataspace.
bool parse_space(const Reader& r, uint64_t at, uint64_t size, std::vector<uint64_t>& shape) {
  r.need(at, std::min<uint64_t>(size, 8));
  const int ver = (uint8_t)r.f[at], rank = (uint8_t)r.f[at + 1];
  uint64_t p;
  if (ver == 1) {
    p = at + 8;
  } else if (ver == 2) {
    const int type = (uint8_t)r.f[at + 3];
    if (type == 2) return false;
    p = at + 4;
  } else {
    throw Error("unsupported dataspace version");
  }
  shape.clear();
  for (int i = 0; i < rank; ++i) shape.push_back(r.len(p + (uint64_t)i * r.sl));
  return true;
}

// Global heap object `index` of the collection at relative address `coll`.
std::string global_heap_object(const Reader& r, uint64_t coll, uint32_t index) {
  const uint64_t at = r.abs(coll);
  if (!r.sig(at, "GCOL")) throw Error("bad global heap collection");
  const uint64_t size = r.len(at + 8);
  uint64_t p = at + 8 + r.sl;
  const uint64_t end = at + size;
  r.need(at, size);
  while (p + 8 + r.sl <= end) {
    const uint32_t idx = (uint32_t)r.le(p, 2);
    const uint64_t osz = r.len(p + 8);
    if (idx == 0) break;  // free space
    if (idx == index) {
      r.need(p + 8 + r.sl, osz);
      return r.f.substr(p + 8 + r.sl, osz);
    }
    p += 8 + r.sl + ((osz + 7) & ~uint64_t(7));
  }
  throw Error("global heap object not found");
}

// Raw element bytes -> Value (byte-swapped to little endian; variable-length
// strings resolved through the global heap into fixed-length ones).
Value make_value(const Reader& r, const Type& t, const std::vector<uint64_t>& shape, const std::string& raw) {
  Value v;
  v.kind = t.kind;
  v.shape = shape;
  if (t.size <= 0 && !t.vlen_string) throw Error("bad datatype size");
  const uint64_t n = elements(shape);
  if (t.vlen_string) {
    const uint64_t esz = 4 + r.so + 4;
    if (raw.size() < checked_bytes(shape, esz)) throw Error("short variable-length string data");
    std::vector<std::string> strs;
    size_t longest = 1;
    for (uint64_t i = 0; i < n; ++i) {
      const uint64_t q = i * esz;
      uint64_t coll = 0;
      for (int k = 0; k < r.so; ++k) coll |= (uint64_t)(uint8_t)raw[q + 4 + k] << (8 * k);
      uint32_t idx = 0, slen = 0;
      for (int k = 0; k < 4; ++k) idx |= (uint32_t)(uint8_t)raw[q + 4 + r.so + k] << (8 * k);
      for (int k = 0; k < 4; ++k) slen |= (uint32_t)(uint8_t)raw[q + k] << (8 * k);
      std::string s = (coll == 0 || slen == 0) ? std::string() : global_heap_object(r, coll, idx);
      if (s.size() > slen) s.resize(slen);
      longest = std::max(longest, s.size());
      strs.push_back(s);
    }
    v.size = (int)longest;
    for (auto& s : strs) {
      s.resize(longest, '\0');
      v.bytes += s;
    }
    return v;
  }
  v.size = t.size;
  if (raw.size() < checked_bytes(shape, (uint64_t)t.size)) throw Error("short element data");
  v.bytes = raw.substr(0, n * (uint64_t)t.size);
  if (t.big_endian && t.size > 1)
    for (uint64_t i = 0; i < n; ++i) std::reverse(v.bytes.begin() + i * t.size, v.bytes.begin() + (i + 1) * t.size);
  return v;
}

Attr parse_attribute(const Reader& r, uint64_t at, uint64_t size) {
  r.need(at, size);
  const int ver = (uint8_t)r.f[at];
  const uint64_t nlen = r.le(at + 2, 2), dlen = r.le(at + 4, 2), slen = r.le(at + 6, 2);
  uint64_t p = at + 8;
  if (ver == 3) p += 1;  // name character set
  else if (ver != 1 && ver != 2) throw Error("unsupported attribute message version");
  auto step = [&](uint64_t n) { return ver == 1 ? ((n + 7) & ~uint64_t(7)) : n; };
  Attr a;
  r.need(p, nlen);
  a.name = std::string(r.f.data() + p, strnlen(r.f.data() + p, nlen));
  p += step(nlen);
  const Type t = parse_type(r, p, dlen);
  p += step(dlen);
  std::vector<uint64_t> shape;
  const bool has = parse_space(r, p, slen, shape);
  p += step(slen);
  if (!has) shape = {0};
  const uint64_t esz = t.vlen_string ? 4 + r.so + 4 : (uint64_t)std::max(t.size, 0);
  const uint64_t bytes = checked_bytes(shape, esz);
  r.need(p, bytes);
  a.value = make_value(r, t, shape, r.f.substr(p, bytes));
  return a;
}

struct Walk {
  const Reader& r;
  std::vector<Object>& out;
  std::set<uint64_t> active;  // object headers on the current path (cycle guard)

  void links_of_symbol_table(uint64_t btree, uint64_t heap, std::vector<std::pair<std::string, uint64_t>>& links,
                             int depth) {
    if (depth > 64) throw Error("group B-tree too deep");
    const uint64_t ha = r.abs(heap);
    if (!r.sig(ha, "HEAP")) throw Error("bad local heap");
    const uint64_t data = r.abs(r.off(ha + 8 + 2 * r.sl));
    const uint64_t dsize = r.len(ha + 8);
    r.need(data, dsize);
    const uint64_t ta = r.abs(btree);
    if (!r.sig(ta, "TREE")) throw Error("bad group B-tree node");
    if ((uint8_t)r.f[ta + 4] != 0) throw Error("not a group B-tree node");
    const int level = (uint8_t)r.f[ta + 5];
    const uint64_t used = r.le(ta + 6, 2);
    uint64_t p = ta + 8 + 2 * r.so + r.sl;  // past key 0
    for (uint64_t i = 0; i < used; ++i, p += r.so + r.sl) {
      const uint64_t child = r.off(p);
      if (level > 0) {
        links_of_symbol_table(child, heap, links, depth + 1);
        continue;
      }
      const uint64_t sa = r.abs(child);
      if (!r.sig(sa, "SNOD")) throw Error("bad symbol table node");
      const uint64_t nsym = r.le(sa + 6, 2);
      const uint64_t esz = 2 * r.so + 8 + 16;
      for (uint64_t k = 0; k < nsym; ++k) {
        const uint64_t e = sa + 8 + k * esz;
        const uint64_t name_off = r.off(e);
        if (name_off >= dsize) throw Error("link name outside the local heap");
        links.push_back({r.cstr(data + name_off), r.off(e + r.so)});
      }
    }
  }

  void object(uint64_t rel, const std::string& name, int parent, int depth) {
    if (depth > 64) throw Error("group nesting deeper than 64 levels");
    const uint64_t at = r.abs(rel);
    if (!active.insert(at).second) return;  // a hard link back up the path
    const std::vector<Msg> msgs = object_messages(r, at);
    Object o;
    o.name = name;
    o.parent = parent;
    bool has_layout = false, has_type = false, has_space = false, space_ok = true;
    Type t;
    std::vector<uint64_t> shape;
    uint64_t btree = kUndef, heap = kUndef;
    std::vector<std::pair<std::string, uint64_t>> links;
    std::string raw;
    bool data_stored = false;
    for (const Msg& m : msgs) {
      switch (m.type) {
        case kMsgDatatype:
          t = parse_type(r, m.at, m.size);
          has_type = true;
          break;
        case kMsgDataspace:
          space_ok = parse_space(r, m.at, m.size, shape);
          has_space = true;
          break;
        case kMsgSymbolTable:
          btree = r.off(m.at);
          heap = r.off(m.at + r.so);
          break;
        case kMsgAttribute:
          o.attrs.push_back(parse_attribute(r, m.at, m.size));
          break;
        case kMsgLinkInfo: {
          const int flags = (uint8_t)r.f[m.at + 1];
          const uint64_t fh = r.off(m.at + 2 + ((flags & 1) ? 8 : 0));
          if (fh != kUndef) throw Error("dense link storage (fractal heap) is not supported");
          break;
        }
        case kMsgLink: {
          const int flags = (uint8_t)r.f[m.at + 1];
          uint64_t p = m.at + 2;
          int ltype = 0;
          if (flags & 0x08) ltype = (uint8_t)r.f[p++];
          if (flags & 0x04) p += 8;
          if (flags & 0x10) p += 1;
          const int nb = 1 << (flags & 3);
          const uint64_t nlen = r.le(p, nb);
          p += nb;
          r.need(p, nlen);
          std::string lname = r.f.substr(p, nlen);
          p += nlen;
          if (ltype == 0) links.push_back({lname, r.off(p)});  // soft / external links are skipped
          break;
        }
        case kMsgLayout: {
          has_layout = true;
          const int ver = (uint8_t)r.f[m.at];
          uint64_t addr = kUndef, size = 0;
          bool stored = false;  // the layout points at data (compact or allocated)
          if (ver == 1 || ver == 2) {
            const int nd = (uint8_t)r.f[m.at + 1], cls = (uint8_t)r.f[m.at + 2];
            uint64_t p = m.at + 8;
            if (cls != 0) {
              addr = r.off(p);
              p += r.so;
            }
            std::vector<uint64_t> dims;
            for (int i = 0; i < nd; ++i) dims.push_back(r.le(p + 4 * i, 4));
            p += 4 * nd;
            if (cls == 0) {
              size = r.le(p, 4);
              r.need(p + 4, size);
              raw = r.f.substr(p + 4, size);
              stored = true;
            } else if (cls == 1) {
              size = checked_bytes(dims, 1);
            } else {
              throw Error("chunked dataset storage is not supported");
            }
          } else if (ver == 3 || ver == 4) {
            const int cls = (uint8_t)r.f[m.at + 1];
            if (cls == 0) {
              size = r.le(m.at + 2, 2);
              r.need(m.at + 4, size);
              raw = r.f.substr(m.at + 4, size);
              stored = true;
            } else if (cls == 1) {
              addr = r.off(m.at + 2);
              size = r.len(m.at + 2 + r.so);
            } else {
              throw Error("chunked or virtual dataset storage is not supported");
            }
          } else {
            throw Error("unsupported layout message version");
          }
          if (addr != kUndef) {
            r.need(r.abs(addr), size);
            raw = r.f.substr(r.abs(addr), size);
            stored = true;
          }
          data_stored = stored;
          break;
        }
        default:
          break;
      }
    }
    const int me = (int)out.size();
    if (has_layout) {
      if (!has_type || !has_space) throw Error("dataset without datatype or dataspace");
      o.is_group = false;
      if (!space_ok) shape = {0};
      const uint64_t esz = t.vlen_string ? 4 + r.so + 4 : (uint64_t)std::max(t.size, 0);
      const uint64_t need = checked_bytes(shape, esz);
      if (raw.size() < need) {
        // Storage that was never allocated reads as the (zero) fill value;
        // allocated storage shorter than the dataspace is corrupt.
        if (data_stored) throw Error("dataset storage smaller than its dataspace");
        if (need > (uint64_t(256) << 20)) throw Error("unallocated dataset too large to materialise");
        raw.resize(need, '\0');
      }
      o.data = make_value(r, t, shape, raw);
      out.push_back(o);
    } else {
      o.is_group = true;
      out.push_back(o);
      if (btree != kUndef) links_of_symbol_table(btree, heap, links, 0);
      std::sort(links.begin(), links.end());
      for (const auto& l : links) object(l.second, l.first, me, depth + 1);
    }
    active.erase(at);
  }
};

}  // namespace

std::string write_file(const std::vector<Object>& objs) {
  if (objs.empty() || !objs[0].is_group || objs[0].parent != -1) throw Error("object 0 must be the root group");
  std::vector<std::vector<int>> kids(objs.size());
  for (size_t i = 1; i < objs.size(); ++i) {
    const int p = objs[i].parent;
    if (p < 0 || p >= (int)i || !objs[p].is_group) throw Error("object " + objs[i].name + ": bad parent");
    kids[p].push_back((int)i);
  }
  Buf f;
  f.zeros(96);  // superblock, written last
  const GroupAt root = write_group(f, objs, kids, 0, 0);
  f.align8();
  Buf sb;
  sb.raw(std::string(kSignature, 8));
  sb.u8(0);  // superblock version
  sb.u8(0);  // free-space storage version
  sb.u8(0);  // root group symbol table entry version
  sb.u8(0);
  sb.u8(0);  // shared header message format version
  sb.u8(8);  // size of offsets
  sb.u8(8);  // size of lengths
  sb.u8(0);
  sb.u16(kLeafK);
  sb.u16(kInternalK);
  sb.u32(0);       // file consistency flags
  sb.u64(0);       // base address
  sb.u64(kUndef);  // free-space info
  sb.u64(f.pos()); // end of file
  sb.u64(kUndef);  // driver info block
  sb.u64(0);       // root entry: link name offset (the empty name)
  sb.u64(root.header);
  sb.u32(1);
  sb.u32(0);
  sb.u64(root.btree);
  sb.u64(root.heap);
  std::memcpy(&f.b[0], sb.b.data(), 96);
  return f.b;
}

std::vector<Object> read_file(const std::string& file) {
  Reader r(file);
  uint64_t sb = kUndef;
  for (uint64_t at = 0; at + 8 <= file.size(); at = at ? at * 2 : 512) {
    if (std::memcmp(file.data() + at, kSignature, 8) == 0) {
      sb = at;
      break;
    }
  }
  if (sb == kUndef) throw Error("not an HDF5 file (no superblock signature)");
  r.need(sb, 16);
  const int ver = (uint8_t)file[sb + 8];
  uint64_t root_header;
  // Addresses are relative to the superblock's position (the user block,
  // if any, precedes it), as libhdf5 resolves them.
  r.base = sb;
  if (ver == 0 || ver == 1) {
    r.so = (uint8_t)file[sb + 13];
    r.sl = (uint8_t)file[sb + 14];
    if ((r.so != 2 && r.so != 4 && r.so != 8) || (r.sl != 2 && r.sl != 4 && r.sl != 8))
      throw Error("unsupported offset or length size");
    const uint64_t p = sb + (ver == 1 ? 28 : 24) + 4 * (uint64_t)r.so;  // root group symbol table entry
    root_header = r.off(p + r.so);
  } else if (ver == 2 || ver == 3) {
    r.so = (uint8_t)file[sb + 9];
    r.sl = (uint8_t)file[sb + 10];
    if ((r.so != 2 && r.so != 4 && r.so != 8) || (r.sl != 2 && r.sl != 4 && r.sl != 8))
      throw Error("unsupported offset or length size");
    root_header = r.off(sb + 12 + 3 * (uint64_t)r.so);
  } else {
    throw Error("unsupported superblock version");
  }
  std::vector<Object> out;
  Walk w{r, out, {}};
  w.object(root_header, "", -1, 0);
  return out;
}

}  // namespace h5
}  // namespace ngl
