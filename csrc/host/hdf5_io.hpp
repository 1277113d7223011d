// Minimal HDF5 file writer and reader (no libhdf5), written from the public
// HDF5 File Format Specification.  It covers the subset that checkpoint
// files need: groups, 1-D/N-D datasets of fixed-size integers, IEEE floats
// and fixed-length strings, and attributes of the same types.
//
// Writer: superblock version 0, version-1 object headers, groups stored as
// symbol tables (version-1 B-tree of group nodes, symbol table nodes, a
// local heap of link names), contiguous dataset storage, fill-value message
// version 2, layout message version 3, attribute messages version 1.  This
// is the layout libhdf5 itself writes by default (its "earliest" format),
// which every HDF5 reader accepts.
//
// Reader: superblock versions 0-3, object headers version 1 and 2 with
// continuation blocks, symbol-table groups (any B-tree depth) and compact
// link-message groups, contiguous and compact layouts (layout messages
// version 1-4), fixed-point / floating-point / fixed-length string types,
// variable-length strings through the global heap, attribute messages
// version 1-3, dataspace messages version 1-2.  Chunked storage and dense
// (fractal-heap) link or attribute storage are reported as unsupported.
//
// The reference writes these files through the hdf5 crate
// (nangila-checkpoint/src/lib.rs:14-133); this is a standalone replacement
// for that path and for h5py in the reference's Python reader
// (python/snippets/read_hdf5_checkpoint.py:21-62).
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace ngl {
namespace h5 {

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// A typed value: kind 'u' / 'i' (little-endian integers), 'f' (IEEE
// little-endian float), 'S' (fixed-length byte string of `size` bytes per
// element).  `shape` empty = scalar.  `bytes` holds prod(shape) elements.
struct Value {
  char kind = 'u';
  int size = 1;
  std::vector<uint64_t> shape;
  std::string bytes;
};

struct Attr {
  std::string name;
  Value value;
};

// One object of a file, in a flat list: objs[0] is the root group
// (parent -1); every other object names its parent group by index.
struct Object {
  bool is_group = true;
  std::string name;
  int parent = -1;
  Value data;  // datasets only
  std::vector<Attr> attrs;
};

// Serialises the object tree to the bytes of an HDF5 file.
std::string write_file(const std::vector<Object>& objs);
// Parses an HDF5 file image (the superblock may follow a user block at
// 0, 512, 1024, 2048, ... bytes) into the flat object list.
std::vector<Object> read_file(const std::string& file);

}  // namespace h5
}  // namespace ngl
