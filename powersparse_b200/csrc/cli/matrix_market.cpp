// Parallel MatrixMarket reader and binary CSR loader of the drop-in CLI
// (interface and accepted format: matrix_market.h).
//
// The reference reads a file twice, line by line with std::getline, strtoll and
// strtod (benchmarks/matrix_market.cpp:97-134).  Here the file is mapped into
// memory and read once by all threads:
//   1. the banner and the size line are read on the calling thread;
//   2. the rest is cut into one chunk of whole lines per thread; each thread
//      parses its lines into (row, column, value) entries in file order (a
//      symmetric off-diagonal entry followed by its mirror), appended to the
//      bucket of the entry's block of rows; numbers go through std::from_chars,
//      and any token from_chars does not take the same way as the C library (a
//      leading '+', hexadecimal floats, overflow) is handed to strtoll / strtod
//      exactly as the reference does;
//   3. one thread per block of rows counts the block's rows, writes their row
//      pointers and places the block's entries, chunk after chunk (so a row keeps
//      file order); a block's stretch of the CSR fits in cache, so these writes
//      stay local.
// Errors: every thread stops at its first malformed record; the problem reported
// is the first one in file order among the declared records, then a wrong record
// count, then the 32-bit capacity limit (the reference checks the capacity while
// it counts, so for a file that both overflows 2^31 - 33 entries and has a
// malformed record after that point it names the capacity first).
#include "matrix_market.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <charconv>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

// The reference's limit on rows, columns, declared and expanded entries.
constexpr long long kLimit = std::numeric_limits<int>::max() - 32;

// Read-only mapping of a regular file (empty files map to nothing).
class MappedFile {
 public:
  explicit MappedFile(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("Cannot open matrix: " + path);
    struct stat st {};
    if (::fstat(fd_, &st) != 0 || !S_ISREG(st.st_mode)) {
      ::close(fd_);
      throw std::runtime_error("Matrix input must be a seekable regular file");
    }
    size_ = size_t(st.st_size);
    if (size_ > 0) {
      void* p = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
      if (p == MAP_FAILED) {
        ::close(fd_);
        throw std::runtime_error("Error reading MatrixMarket input");
      }
      ::madvise(p, size_, MADV_SEQUENTIAL);
      data_ = static_cast<const char*>(p);
    }
  }
  ~MappedFile() {
    if (data_) ::munmap(const_cast<char*>(data_), size_);
    if (fd_ >= 0) ::close(fd_);
  }
  MappedFile(const MappedFile&) = delete;
  MappedFile& operator=(const MappedFile&) = delete;
  const char* begin() const { return data_; }
  const char* end() const { return data_ + size_; }
  size_t size() const { return size_; }

 private:
  int fd_ = -1;
  const char* data_ = nullptr;
  size_t size_ = 0;
};

// One line of the file: [text, stop) is what the reference's reader sees of it
// (std::getline drops the '\n', c_str() ends the text at the first '\0').
struct Line {
  const char* text;
  const char* stop;
};

inline bool blank(char c) { return c == ' ' || c == '\t' || c == '\r' || c == '\f' || c == '\v' || c == '\n'; }

// The line starting at `p` (< `end`); `next` receives the start of the line after.
inline Line line_at(const char* p, const char* end, const char** next) {
  const char* nl = static_cast<const char*>(std::memchr(p, '\n', size_t(end - p)));
  const char* le = nl ? nl : end;
  *next = nl ? nl + 1 : end;
  const char* z = static_cast<const char*>(std::memchr(p, '\0', size_t(le - p)));
  return {p, z ? z : le};
}

// A data line holds a record: neither blank nor a '%' comment.
inline bool is_record(const Line& l) {
  const char* p = l.text;
  while (p < l.stop && blank(*p)) ++p;
  return p < l.stop && *p != '%';
}

enum class Fault { kNone, kInteger, kRange, kValue, kExtra };

const char* fault_text(Fault f) {
  switch (f) {
    case Fault::kInteger: return "Invalid integer in MatrixMarket input";
    case Fault::kRange: return "MatrixMarket index outside the declared dimensions";
    case Fault::kValue: return "Invalid finite FP32 value in MatrixMarket input";
    case Fault::kExtra: return "Unexpected extra fields in MatrixMarket record";
    default: return "";
  }
}

// Field scanner over one line's text, with the reference's token rules: a number
// may be preceded by blanks and must be followed by a blank or the end of the text.
class Fields {
 public:
  explicit Fields(const Line& l) : p_(l.text), stop_(l.stop) {}

  bool integer(long long* out) {
    skip();
    long long v = 0;
    const auto r = std::from_chars(p_, stop_, v);
    if (r.ec == std::errc() && (r.ptr == stop_ || blank(*r.ptr))) {
      p_ = r.ptr;
      *out = v;
      return true;
    }
    // Everything else takes the C library's path (strtoll, base 10).
    const std::string tok(p_, stop_);
    char* e = nullptr;
    errno = 0;
    v = std::strtoll(tok.c_str(), &e, 10);
    if (e == tok.c_str() || errno == ERANGE || (*e && !blank(*e))) return false;
    p_ += e - tok.c_str();
    *out = v;
    return true;
  }

  bool real(float* out) {
    skip();
    double d = 0;
    const auto r = std::from_chars(p_, stop_, d);
    if (r.ec == std::errc() && (r.ptr == stop_ || blank(*r.ptr))) {
      p_ = r.ptr;
    } else {
      // strtod, as the reference: signs, hexadecimal floats, under/overflow.
      const std::string tok(p_, stop_);
      char* e = nullptr;
      d = std::strtod(tok.c_str(), &e);
      if (e == tok.c_str() || (*e && !blank(*e))) return false;
      p_ += e - tok.c_str();
    }
    if (!std::isfinite(d) || std::abs(d) > std::numeric_limits<float>::max()) return false;
    *out = static_cast<float>(d);
    return true;
  }

  bool at_end() {
    skip();
    return p_ == stop_;
  }

 private:
  void skip() {
    while (p_ < stop_ && blank(*p_)) ++p_;
  }
  const char* p_;
  const char* stop_;
};

enum class Field { kPattern, kReal, kInteger };

struct Shape {
  long long rows, cols, entries;
  Field field;
  bool symmetric;
};

// Banner (first line) and size line; returns the start of the first entry line.
const char* read_header(const MappedFile& f, Shape* shape) {
  const char* p = f.begin();
  const char* end = f.end();
  if (f.size() == 0) throw std::runtime_error("Empty MatrixMarket file");
  const char* next = nullptr;
  const char* nl = static_cast<const char*>(std::memchr(p, '\n', f.size()));
  const std::string banner_line(p, nl ? nl : end);
  next = nl ? nl + 1 : end;
  std::istringstream banner(banner_line);
  std::string magic, object, format, field, symmetry, more;
  if (!(banner >> magic >> object >> format >> field >> symmetry) || (banner >> more) ||
      magic != "%%MatrixMarket" || object != "matrix" || format != "coordinate" ||
      (field != "pattern" && field != "real" && field != "integer") ||
      (symmetry != "general" && symmetry != "symmetric"))
    throw std::runtime_error("Expected MatrixMarket coordinate pattern/real/integer general/symmetric");
  shape->field = field == "pattern" ? Field::kPattern : field == "real" ? Field::kReal : Field::kInteger;
  shape->symmetric = symmetry == "symmetric";
  p = next;
  while (p < end) {
    const Line l = line_at(p, end, &next);
    p = next;
    if (!is_record(l)) continue;
    Fields fs(l);
    if (!fs.integer(&shape->rows) || !fs.integer(&shape->cols) || !fs.integer(&shape->entries))
      throw std::runtime_error(fault_text(Fault::kInteger));
    if (!fs.at_end()) throw std::runtime_error(fault_text(Fault::kExtra));
    if (shape->rows <= 0 || shape->cols <= 0 || shape->entries <= 0 || shape->rows > kLimit ||
        shape->cols > kLimit || shape->entries > kLimit || (shape->symmetric && shape->rows != shape->cols))
      throw std::runtime_error("Matrix must be nonempty and fit 32-bit CSR indices");
    return p;
  }
  throw std::runtime_error("Missing MatrixMarket dimensions");
}

struct Entry {
  int row, col;
  float value;
};

// Rows are cut into blocks of 2^kBlockShift rows; entries are appended to the
// bucket of their row's block while they are parsed, so the final placement
// writes one block's stretch of the CSR at a time.
struct Blocking {
  int shift;
  int count;
  explicit Blocking(long long rows) {
    shift = 12;
    while ((rows >> shift) > 4096) ++shift;
    count = int(((rows - 1) >> shift) + 1);
  }
};

// What one thread parsed from its chunk of lines.
struct Chunk {
  const char* begin = nullptr;
  const char* end = nullptr;
  std::vector<std::vector<Entry>> buckets;  // per row block, in file order (mirrors right after their entry)
  long long records = 0;                    // records parsed before the first fault (all of them without one)
  long long emitted = 0;                    // entries appended
  Fault fault = Fault::kNone;               // first malformed record of the chunk, record index `records`
};

void parse_chunk(const Shape& shape, const Blocking& blk, Chunk& c) {
  c.buckets.assign(size_t(blk.count), {});
  // About 25 bytes of text per record; row labels spread the entries over the blocks.
  const size_t guess = size_t(c.end - c.begin) / 25 * (shape.symmetric ? 2 : 1) / size_t(blk.count);
  for (auto& b : c.buckets) b.reserve(guess + guess / 4 + 16);
  // Without a NUL byte in the chunk (the usual case) a line's text ends at its '\n'.
  const bool nul = std::memchr(c.begin, '\0', size_t(c.end - c.begin)) != nullptr;
  const char* p = c.begin;
  while (p < c.end) {
    Line l;
    const char* nl = static_cast<const char*>(std::memchr(p, '\n', size_t(c.end - p)));
    const char* next = nl ? nl + 1 : c.end;
    if (nul) {
      l = line_at(p, c.end, &next);
    } else {
      l = {p, nl ? nl : c.end};
    }
    p = next;
    if (!is_record(l)) continue;
    Fields fs(l);
    long long row = 0, col = 0;
    if (!fs.integer(&row) || !fs.integer(&col)) {
      c.fault = Fault::kInteger;
      return;
    }
    if (row < 1 || row > shape.rows || col < 1 || col > shape.cols) {
      c.fault = Fault::kRange;
      return;
    }
    float value = 1.0f;
    if (shape.field == Field::kInteger) {
      long long v = 0;
      if (!fs.integer(&v)) {
        c.fault = Fault::kInteger;
        return;
      }
      value = static_cast<float>(v);
    } else if (shape.field == Field::kReal) {
      if (!fs.real(&value)) {
        c.fault = Fault::kValue;
        return;
      }
    }
    if (!fs.at_end()) {
      c.fault = Fault::kExtra;
      return;
    }
    const int r = int(row - 1), k = int(col - 1);
    c.buckets[size_t(r >> blk.shift)].push_back({r, k, value});
    ++c.emitted;
    if (shape.symmetric && r != k) {
      c.buckets[size_t(k >> blk.shift)].push_back({k, r, value});
      ++c.emitted;
    }
    ++c.records;
  }
}

// Runs body(i) for i in [0, n) on up to `threads` threads (the calling one included).
template <typename Body>
void parallel_for(int n, int threads, Body body) {
  std::vector<std::thread> pool;
  const int t = std::max(1, std::min(n, threads));
  for (int w = 1; w < t; ++w)
    pool.emplace_back([&, w] {
      for (int i = w; i < n; i += t) body(i);
    });
  for (int i = 0; i < n; i += t) body(i);
  for (auto& th : pool) th.join();
}

CsrMatrix read_text(const std::string& path, int threads, long long min_chunk) {
  const MappedFile file(path);
  Shape shape{};
  const char* data = read_header(file, &shape);
  const char* end = file.end();

  // Chunks of whole lines, at least `min_chunk` bytes each.
  const size_t bytes = size_t(end - data);
  const int workers = threads > 0 ? threads : int(std::max(1u, std::thread::hardware_concurrency()));
  const int parts = int(std::min<size_t>(size_t(workers), std::max<size_t>(1, bytes / size_t(std::max(1LL, min_chunk)))));
  std::vector<Chunk> chunks(static_cast<size_t>(parts));
  const char* cut = data;
  for (int i = 0; i < parts; ++i) {
    chunks[i].begin = cut;
    const char* target = i + 1 == parts ? end : data + bytes / parts * (i + 1);
    if (target < cut) target = cut;
    const char* nl = target < end ? static_cast<const char*>(std::memchr(target, '\n', size_t(end - target)))
                                  : nullptr;
    cut = i + 1 == parts ? end : (nl ? nl + 1 : end);
    chunks[i].end = cut;
  }
  const Blocking blk(shape.rows);
  parallel_for(parts, parts, [&](int i) { parse_chunk(shape, blk, chunks[size_t(i)]); });

  // The first fault in file order among the declared records, then the record count.
  long long seen = 0;
  for (const Chunk& c : chunks) {
    if (c.fault != Fault::kNone) {
      if (seen + c.records < shape.entries) throw std::runtime_error(fault_text(c.fault));
      throw std::runtime_error("More entries than declared in MatrixMarket input");
    }
    seen += c.records;
  }
  if (seen < shape.entries) throw std::runtime_error("Truncated MatrixMarket input");
  if (seen > shape.entries) throw std::runtime_error("More entries than declared in MatrixMarket input");
  long long expanded = 0;
  for (const Chunk& c : chunks) expanded += c.emitted;
  if (expanded > kLimit) throw std::runtime_error("Expanded matrix exceeds 32-bit CSR capacity");

  CsrMatrix m;
  m.rows = int(shape.rows);
  m.cols = int(shape.cols);
  m.row_ptr.resize(size_t(m.rows) + 1);  // every element is written below (by the block's thread)
  m.col_ind.resize(size_t(expanded));
  m.values.resize(size_t(expanded));
  // Block b's stretch of the CSR starts after the entries of blocks < b.
  std::vector<long long> block_start(static_cast<size_t>(blk.count) + 1, 0);
  for (int b = 0; b < blk.count; ++b) {
    long long n = 0;
    for (const Chunk& c : chunks) n += (long long)c.buckets[size_t(b)].size();
    block_start[size_t(b) + 1] = block_start[size_t(b)] + n;
  }
  // Per block: row counts, row pointers, then the entries of every chunk in chunk
  // order (so each row keeps file order).
  parallel_for(blk.count, workers, [&](int b) {
    const long long r0 = (long long)b << blk.shift;
    const long long r1 = std::min<long long>(m.rows, (long long)(b + 1) << blk.shift);
    std::vector<long long> cursor(static_cast<size_t>(r1 - r0) + 1, 0);
    for (const Chunk& c : chunks)
      for (const Entry& e : c.buckets[size_t(b)]) ++cursor[size_t(e.row - r0) + 1];
    cursor[0] = block_start[size_t(b)];
    for (long long r = r0; r < r1; ++r) {
      cursor[size_t(r - r0) + 1] += cursor[size_t(r - r0)];
      m.row_ptr[size_t(r)] = int(cursor[size_t(r - r0)]);
    }
    for (Chunk& c : chunks) {
      for (const Entry& e : c.buckets[size_t(b)]) {
        const long long at = cursor[size_t(e.row - r0)]++;
        m.col_ind[size_t(at)] = e.col;
        m.values[size_t(at)] = e.value;
      }
      std::vector<Entry>().swap(c.buckets[size_t(b)]);
    }
  });
  m.row_ptr[size_t(m.rows)] = int(expanded);
  return m;
}

// Binary CSR written by powersparse_b200.synth.write_csr_bin.
CsrMatrix read_binary(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("Cannot open matrix: " + path);
  char magic[8];
  long long dims[3];
  in.read(magic, 8);
  in.read(reinterpret_cast<char*>(dims), sizeof(dims));
  if (!in || std::memcmp(magic, "PSCSR001", 8) != 0) throw std::runtime_error("Bad binary CSR header: " + path);
  if (dims[0] <= 0 || dims[1] <= 0 || dims[2] <= 0 || dims[0] > kLimit || dims[1] > kLimit || dims[2] > kLimit)
    throw std::runtime_error("Matrix must be nonempty and fit 32-bit CSR indices");
  CsrMatrix m;
  m.rows = int(dims[0]);
  m.cols = int(dims[1]);
  m.row_ptr.resize(size_t(m.rows) + 1);
  m.col_ind.resize(size_t(dims[2]));
  m.values.resize(size_t(dims[2]));
  in.read(reinterpret_cast<char*>(m.row_ptr.data()), std::streamsize(4 * m.row_ptr.size()));
  in.read(reinterpret_cast<char*>(m.col_ind.data()), std::streamsize(4 * m.col_ind.size()));
  in.read(reinterpret_cast<char*>(m.values.data()), std::streamsize(4 * m.values.size()));
  if (!in) throw std::runtime_error("Truncated binary CSR: " + path);
  return m;
}

bool has_binary_magic(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  char magic[8] = {};
  return in.read(magic, 8) && std::memcmp(magic, "PSCSR001", 8) == 0;
}

}  // namespace

CsrMatrix ReadMatrixMarketChunked(const std::string& path, int threads, long long min_chunk_bytes) {
  if (has_binary_magic(path)) return read_binary(path);
  return read_text(path, threads, min_chunk_bytes);
}

CsrMatrix ReadMatrixMarket(const std::string& path, int threads) {
  return ReadMatrixMarketChunked(path, threads, 4LL << 20);
}
