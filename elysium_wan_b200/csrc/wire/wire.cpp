// Native data-plane codecs and frame I/O for the TCP (WAN) transport.
//
// Reference behaviour: src/wantrain/codec/planes.py (byte-plane split plus an
// entropy coder; zlib container here, which the reference's decoder also
// accepts), codec/fp8_planes.py (sign+exponent / mantissa nibble planes),
// codec/f32_planes.py (plane-major fp32 bytes) and transport/framing.py (the
// frame header). The payload layouts and the header are kept byte-compatible
// so a frame written by one side decodes on the other; the implementation is
// C++ with the planes compressed on parallel threads and every socket call
// made with the interpreter lock released.
//
// Frame (little-endian): magic u16 0xE17A | type u8 | codec u8 | step u32 |
// mb u32 | chunk u16 | ndim u8 | frag_idx u16 | frag_cnt u16 | dims u32 x ndim
// | paylen u64 | payload.
#include <errno.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/socket.h>
#include <sys/uio.h>
#include <zlib.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace py = pybind11;

namespace {

constexpr uint16_t kMagic = 0xE17A;

// ------------------------------------------------------------------ zlib
std::string deflate_bytes(const uint8_t* p, size_t n, int level) {
  uLongf cap = compressBound(static_cast<uLong>(n));
  std::string out(cap, '\0');
  int rc = compress2(reinterpret_cast<Bytef*>(&out[0]), &cap, p, static_cast<uLong>(n), level);
  if (rc != Z_OK) throw std::runtime_error("zlib compress failed");
  out.resize(cap);
  return out;
}

std::string inflate_bytes(const uint8_t* p, size_t n, size_t expect) {
  // zstd containers (the reference's preferred coder) are not decodable here.
  if (n >= 4 && p[0] == 0x28 && p[1] == 0xb5 && p[2] == 0x2f && p[3] == 0xfd)
    throw std::runtime_error("payload is zstd-compressed; this build decodes zlib containers");
  std::string out(expect, '\0');
  z_stream zs{};
  if (inflateInit(&zs) != Z_OK) throw std::runtime_error("zlib init failed");
  zs.next_in = const_cast<Bytef*>(p);
  zs.avail_in = static_cast<uInt>(n);
  zs.next_out = reinterpret_cast<Bytef*>(&out[0]);
  zs.avail_out = static_cast<uInt>(expect);
  const int rc = inflate(&zs, Z_FINISH);
  const size_t got = expect - zs.avail_out;
  inflateEnd(&zs);
  if (rc != Z_STREAM_END || got != expect) throw std::runtime_error("zlib stream is corrupt");
  return out;
}

// One zlib stream compressed on several threads (the method of pigz, by Mark
// Adler): the input is cut into blocks; each block is raw-deflated on its own
// thread, primed with the previous 32 KiB as its dictionary, and ended with a
// sync flush (the last with a finish), so the concatenated blocks form one
// valid deflate stream; the zlib header and the Adler-32 of the whole input
// (combined from the blocks' checksums) wrap it. Any zlib inflater decodes it.
constexpr size_t kBlock = 1 << 20;
constexpr size_t kDict = 32768;

std::string deflate_stream_mt(const uint8_t* p, size_t n, int level, int threads) {
  if (n <= kBlock || threads <= 1) return deflate_bytes(p, n, level);
  const size_t nblk = (n + kBlock - 1) / kBlock;
  std::vector<std::string> blk(nblk);
  std::vector<uLong> ad(nblk);
  std::vector<std::string> err(nblk);
  std::atomic<size_t> next{0};
  auto work = [&] {
    for (size_t b = next.fetch_add(1); b < nblk; b = next.fetch_add(1)) {
      const size_t lo = b * kBlock, len = std::min(kBlock, n - lo);
      z_stream zs{};
      if (deflateInit2(&zs, level, Z_DEFLATED, -15, 8, Z_DEFAULT_STRATEGY) != Z_OK) {
        err[b] = "deflateInit2 failed";
        continue;
      }
      if (b > 0) {
        const size_t dl = std::min(kDict, lo);
        deflateSetDictionary(&zs, p + lo - dl, static_cast<uInt>(dl));
      }
      std::string out(deflateBound(&zs, static_cast<uLong>(len)) + 16, '\0');
      zs.next_in = const_cast<Bytef*>(p + lo);
      zs.avail_in = static_cast<uInt>(len);
      zs.next_out = reinterpret_cast<Bytef*>(&out[0]);
      zs.avail_out = static_cast<uInt>(out.size());
      const int rc = deflate(&zs, b + 1 == nblk ? Z_FINISH : Z_SYNC_FLUSH);
      if ((b + 1 == nblk && rc != Z_STREAM_END) || (b + 1 < nblk && rc != Z_OK)) err[b] = "deflate failed";
      out.resize(out.size() - zs.avail_out);
      deflateEnd(&zs);
      blk[b] = std::move(out);
      ad[b] = adler32(adler32(0L, Z_NULL, 0), p + lo, static_cast<uInt>(len));
    }
  };
  std::vector<std::thread> th;
  const int nt = static_cast<int>(std::min<size_t>(threads, nblk));
  for (int i = 0; i < nt; ++i) th.emplace_back(work);
  for (auto& t : th) t.join();
  for (auto& e : err)
    if (!e.empty()) throw std::runtime_error(e);
  uLong a = ad[0];
  for (size_t b = 1; b < nblk; ++b)
    a = adler32_combine(a, ad[b], static_cast<z_off_t>(std::min(kBlock, n - b * kBlock)));
  std::string out;
  out.push_back(static_cast<char>(0x78));
  out.push_back(static_cast<char>(level <= 1 ? 0x01 : 0x9c));
  for (auto& b : blk) out += b;
  for (int sh = 24; sh >= 0; sh -= 8) out.push_back(static_cast<char>((a >> sh) & 0xff));
  return out;
}

int g_threads = 0;  // 0 = hardware concurrency

int codec_threads() {
  if (g_threads > 0) return g_threads;
  const unsigned h = std::thread::hardware_concurrency();
  return h ? static_cast<int>(h) : 4;
}

// Compress each piece (an independent plane) as one zlib stream, the pieces'
// blocks sharing the thread budget.
std::vector<std::string> deflate_parallel(const std::vector<std::string>& pieces, int level) {
  std::vector<std::string> out(pieces.size());
  const int per = std::max(1, codec_threads() / static_cast<int>(pieces.size()));
  std::vector<std::thread> th;
  std::vector<std::string> err(pieces.size());
  for (size_t i = 0; i < pieces.size(); ++i) {
    th.emplace_back([&, i] {
      try {
        out[i] = deflate_stream_mt(reinterpret_cast<const uint8_t*>(pieces[i].data()),
                                   pieces[i].size(), level, per);
      } catch (const std::exception& e) {
        err[i] = e.what();
      }
    });
  }
  for (auto& t : th) t.join();
  for (auto& e : err)
    if (!e.empty()) throw std::runtime_error(e);
  return out;
}

template <typename T>
void put(std::string& s, T v) {
  s.append(reinterpret_cast<const char*>(&v), sizeof(T));
}

template <typename T>
T get(const uint8_t* p, size_t n, size_t& off) {
  if (off + sizeof(T) > n) throw std::runtime_error("payload truncated");
  T v;
  std::memcpy(&v, p + off, sizeof(T));
  off += sizeof(T);
  return v;
}

py::buffer_info as_bytes(const py::buffer& b) {
  py::buffer_info info = b.request();
  return info;
}

// ------------------------------------------------------------------ planes
// Header <BBQ: dtype id, plane count, element count; then u32 blob sizes;
// then the blobs. Elements of esz > 1 bytes split into esz planes, most
// significant byte first; one-byte elements go as one interleaved blob.
py::bytes planes_encode(py::buffer data, int esz, int dtype_id, int level) {
  auto info = as_bytes(data);
  const uint8_t* p = static_cast<const uint8_t*>(info.ptr);
  const size_t nbytes = static_cast<size_t>(info.size) * info.itemsize;
  if (esz < 1 || esz > 8 || nbytes % esz) throw std::invalid_argument("planes: bad element size");
  const size_t n = nbytes / esz;
  std::vector<std::string> pieces;
  {
    py::gil_scoped_release nogil;
    if (esz == 1) {
      pieces.emplace_back(reinterpret_cast<const char*>(p), nbytes);
    } else {
      pieces.resize(esz);
      for (int k = 0; k < esz; ++k) pieces[k].resize(n);
      for (size_t i = 0; i < n; ++i)
        for (int k = 0; k < esz; ++k) pieces[k][i] = static_cast<char>(p[i * esz + (esz - 1 - k)]);
    }
    pieces = deflate_parallel(pieces, level);
  }
  std::string out;
  put<uint8_t>(out, static_cast<uint8_t>(dtype_id));
  put<uint8_t>(out, static_cast<uint8_t>(pieces.size()));
  put<uint64_t>(out, static_cast<uint64_t>(n));
  for (auto& b : pieces) put<uint32_t>(out, static_cast<uint32_t>(b.size()));
  for (auto& b : pieces) out += b;
  return py::bytes(out);
}

// -> (dtype id, element size, raw little-endian element bytes)
py::tuple planes_decode(py::buffer payload, int esz) {
  auto info = as_bytes(payload);
  const uint8_t* p = static_cast<const uint8_t*>(info.ptr);
  const size_t n_in = static_cast<size_t>(info.size) * info.itemsize;
  size_t off = 0;
  const int did = get<uint8_t>(p, n_in, off);
  const int np_ = get<uint8_t>(p, n_in, off);
  const uint64_t n = get<uint64_t>(p, n_in, off);
  std::vector<uint32_t> sizes(np_);
  for (int i = 0; i < np_; ++i) sizes[i] = get<uint32_t>(p, n_in, off);
  if (np_ != 1 && np_ != esz) throw std::runtime_error("planes: plane count does not match dtype");
  std::string raw;
  {
    py::gil_scoped_release nogil;
    if (np_ == 1) {
      if (off + sizes[0] > n_in) throw std::runtime_error("payload truncated");
      raw = inflate_bytes(p + off, sizes[0], n * esz);
    } else {
      // planes inflate on parallel threads
      raw.assign(n * esz, '\0');
      std::vector<size_t> offs(np_);
      for (int k = 0; k < np_; ++k) {
        if (off + sizes[k] > n_in) throw std::runtime_error("payload truncated");
        offs[k] = off;
        off += sizes[k];
      }
      std::vector<std::string> err(np_);
      std::vector<std::thread> th;
      for (int k = 0; k < np_; ++k) {
        th.emplace_back([&, k] {
          try {
            std::string plane = inflate_bytes(p + offs[k], sizes[k], n);
            for (size_t i = 0; i < n; ++i) raw[i * esz + (esz - 1 - k)] = plane[i];
          } catch (const std::exception& e) {
            err[k] = e.what();
          }
        });
      }
      for (auto& t : th) t.join();
      for (auto& e : err)
        if (!e.empty()) throw std::runtime_error(e);
    }
  }
  return py::make_tuple(did, esz, py::bytes(raw));
}

// Two planes in one payload, each zlib-compressed: a bytes plane (for example
// e4m3 codes) and a second blob (for example its fp32 block scales, split
// most significant byte first). Header <BBQ with dtype id, 2, element count.
py::bytes pair_encode(py::buffer a, py::buffer b, int b_esz, int dtype_id, int level) {
  auto ia = as_bytes(a), ib = as_bytes(b);
  const uint8_t* pa = static_cast<const uint8_t*>(ia.ptr);
  const uint8_t* pb = static_cast<const uint8_t*>(ib.ptr);
  const size_t na = static_cast<size_t>(ia.size) * ia.itemsize;
  const size_t nb = static_cast<size_t>(ib.size) * ib.itemsize;
  if (nb % b_esz) throw std::invalid_argument("pair: bad second element size");
  std::vector<std::string> pieces(2);
  {
    py::gil_scoped_release nogil;
    pieces[0].assign(reinterpret_cast<const char*>(pa), na);
    const size_t m = nb / b_esz;
    pieces[1].resize(nb);
    for (int k = 0; k < b_esz; ++k)
      for (size_t i = 0; i < m; ++i) pieces[1][k * m + i] = static_cast<char>(pb[i * b_esz + (b_esz - 1 - k)]);
    pieces = deflate_parallel(pieces, level);
  }
  std::string out;
  put<uint8_t>(out, static_cast<uint8_t>(dtype_id));
  put<uint8_t>(out, 2);
  put<uint64_t>(out, static_cast<uint64_t>(na));
  put<uint32_t>(out, static_cast<uint32_t>(pieces[0].size()));
  put<uint32_t>(out, static_cast<uint32_t>(pieces[1].size()));
  put<uint64_t>(out, static_cast<uint64_t>(nb));
  out += pieces[0];
  out += pieces[1];
  return py::bytes(out);
}

py::tuple pair_decode(py::buffer payload, int b_esz) {
  auto info = as_bytes(payload);
  const uint8_t* p = static_cast<const uint8_t*>(info.ptr);
  const size_t n_in = static_cast<size_t>(info.size) * info.itemsize;
  size_t off = 0;
  const int did = get<uint8_t>(p, n_in, off);
  if (get<uint8_t>(p, n_in, off) != 2) throw std::runtime_error("pair: expected two planes");
  const uint64_t na = get<uint64_t>(p, n_in, off);
  const uint32_t s0 = get<uint32_t>(p, n_in, off), s1 = get<uint32_t>(p, n_in, off);
  const uint64_t nb = get<uint64_t>(p, n_in, off);
  if (off + s0 + s1 > n_in || nb % b_esz) throw std::runtime_error("payload truncated");
  std::string a, b;
  {
    py::gil_scoped_release nogil;
    a = inflate_bytes(p + off, s0, na);
    std::string planes = inflate_bytes(p + off + s0, s1, nb);
    b.assign(nb, '\0');
    const size_t m = nb / b_esz;
    for (int k = 0; k < b_esz; ++k)
      for (size_t i = 0; i < m; ++i) b[i * b_esz + (b_esz - 1 - k)] = planes[k * m + i];
  }
  return py::make_tuple(did, py::bytes(a), py::bytes(b));
}

// ------------------------------------------------------------------ fp8 nibble planes
// <QII: element count, compressed hi size, compressed lo size; hi = sign and
// exponent nibbles, lo = mantissa nibbles, two per byte (first element in the
// high half).
py::bytes fp8_planes_encode(py::buffer codes, int level) {
  auto info = as_bytes(codes);
  const uint8_t* p = static_cast<const uint8_t*>(info.ptr);
  const size_t n = static_cast<size_t>(info.size) * info.itemsize;
  std::vector<std::string> pieces(2);
  {
    py::gil_scoped_release nogil;
    const size_t m = (n + 1) / 2;
    pieces[0].assign(m, '\0');
    pieces[1].assign(m, '\0');
    for (size_t i = 0; i < n; ++i) {
      const int sh = (i & 1) ? 0 : 4;
      pieces[0][i / 2] |= static_cast<char>((p[i] >> 4) << sh);
      pieces[1][i / 2] |= static_cast<char>((p[i] & 0x0F) << sh);
    }
    pieces = deflate_parallel(pieces, level);
  }
  std::string out;
  put<uint64_t>(out, static_cast<uint64_t>(n));
  put<uint32_t>(out, static_cast<uint32_t>(pieces[0].size()));
  put<uint32_t>(out, static_cast<uint32_t>(pieces[1].size()));
  out += pieces[0];
  out += pieces[1];
  return py::bytes(out);
}

py::bytes fp8_planes_decode(py::buffer payload) {
  auto info = as_bytes(payload);
  const uint8_t* p = static_cast<const uint8_t*>(info.ptr);
  const size_t n_in = static_cast<size_t>(info.size) * info.itemsize;
  size_t off = 0;
  const uint64_t n = get<uint64_t>(p, n_in, off);
  const uint32_t nhi = get<uint32_t>(p, n_in, off), nlo = get<uint32_t>(p, n_in, off);
  if (off + nhi + nlo > n_in) throw std::runtime_error("payload truncated");
  std::string out(n, '\0');
  {
    py::gil_scoped_release nogil;
    const size_t m = (n + 1) / 2;
    std::string hi = inflate_bytes(p + off, nhi, m), lo = inflate_bytes(p + off + nhi, nlo, m);
    for (size_t i = 0; i < n; ++i) {
      const int sh = (i & 1) ? 0 : 4;
      const uint8_t h = (static_cast<uint8_t>(hi[i / 2]) >> sh) & 0x0F;
      const uint8_t l = (static_cast<uint8_t>(lo[i / 2]) >> sh) & 0x0F;
      out[i] = static_cast<char>((h << 4) | l);
    }
  }
  return py::bytes(out);
}

// ------------------------------------------------------------------ f32 planes
// <Q element count + one zlib blob of the plane-major bytes (all byte 0s,
// then all byte 1s, ... in memory order).
py::bytes f32_planes_encode(py::buffer data, int level) {
  auto info = as_bytes(data);
  const uint8_t* p = static_cast<const uint8_t*>(info.ptr);
  const size_t nbytes = static_cast<size_t>(info.size) * info.itemsize;
  if (nbytes % 4) throw std::invalid_argument("f32 planes: not fp32 data");
  const size_t n = nbytes / 4;
  std::string comp;
  {
    py::gil_scoped_release nogil;
    std::string planes(nbytes, '\0');
    for (size_t i = 0; i < n; ++i)
      for (int k = 0; k < 4; ++k) planes[k * n + i] = static_cast<char>(p[i * 4 + k]);
    comp = deflate_stream_mt(reinterpret_cast<const uint8_t*>(planes.data()), planes.size(), level,
                             codec_threads());
  }
  std::string out;
  put<uint64_t>(out, static_cast<uint64_t>(n));
  out += comp;
  return py::bytes(out);
}

py::bytes f32_planes_decode(py::buffer payload) {
  auto info = as_bytes(payload);
  const uint8_t* p = static_cast<const uint8_t*>(info.ptr);
  const size_t n_in = static_cast<size_t>(info.size) * info.itemsize;
  size_t off = 0;
  const uint64_t n = get<uint64_t>(p, n_in, off);
  std::string out(n * 4, '\0');
  {
    py::gil_scoped_release nogil;
    std::string planes = inflate_bytes(p + off, n_in - off, n * 4);
    for (size_t i = 0; i < n; ++i)
      for (int k = 0; k < 4; ++k) out[i * 4 + k] = planes[k * n + i];
  }
  return py::bytes(out);
}

// ------------------------------------------------------------------ frame I/O
#pragma pack(push, 1)
struct Header {
  uint16_t magic;
  uint8_t type, codec;
  uint32_t step, mb;
  uint16_t chunk;
  uint8_t ndim;
  uint16_t frag_idx, frag_cnt;
};
#pragma pack(pop)
static_assert(sizeof(Header) == 19, "frame header is 19 bytes");

std::string pack_header(int type, int codec, uint32_t step, uint32_t mb, int chunk,
                        const std::vector<uint32_t>& shape, int frag_idx, int frag_cnt,
                        uint64_t paylen) {
  if (shape.size() > 255) throw std::invalid_argument("frame: ndim > 255");
  Header h{kMagic, static_cast<uint8_t>(type), static_cast<uint8_t>(codec), step, mb,
           static_cast<uint16_t>(chunk), static_cast<uint8_t>(shape.size()),
           static_cast<uint16_t>(frag_idx), static_cast<uint16_t>(frag_cnt)};
  std::string s(reinterpret_cast<const char*>(&h), sizeof(h));
  for (uint32_t d : shape) put<uint32_t>(s, d);
  put<uint64_t>(s, paylen);
  return s;
}

// Write header + payload with writev; -> bytes sent. Raises on a socket error.
size_t send_frame(int fd, int type, int codec, uint32_t step, uint32_t mb, int chunk,
                  std::vector<uint32_t> shape, py::buffer payload, int frag_idx, int frag_cnt) {
  auto info = payload.request();
  const char* p = static_cast<const char*>(info.ptr);
  const size_t n = static_cast<size_t>(info.size) * info.itemsize;
  std::string hdr = pack_header(type, codec, step, mb, chunk, shape, frag_idx, frag_cnt, n);
  size_t sent_h = 0, sent_p = 0;
  bool stalled = false;
  std::chrono::steady_clock::time_point stall_start;
  long backoff_us = 1000;
  py::gil_scoped_release nogil;
  while (sent_h < hdr.size() || sent_p < n) {
    iovec iov[2];
    int cnt = 0;
    if (sent_h < hdr.size()) {
      iov[cnt].iov_base = const_cast<char*>(hdr.data()) + sent_h;
      iov[cnt++].iov_len = hdr.size() - sent_h;
    }
    if (sent_p < n) {
      iov[cnt].iov_base = const_cast<char*>(p) + sent_p;
      iov[cnt++].iov_len = n - sent_p;
    }
    msghdr mh{};
    mh.msg_iov = iov;
    mh.msg_iovlen = cnt;
    const ssize_t w = sendmsg(fd, &mh, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      // The kernel refused for lack of buffer space or would block: nothing
      // was written, so the same bytes go again after a backoff (1 ms
      // doubling to 100 ms); 5 s without progress raises the last error.
      if (errno == ENOBUFS || errno == EAGAIN || errno == EWOULDBLOCK) {
        const auto now = std::chrono::steady_clock::now();
        if (!stalled) {
          stalled = true;
          stall_start = now;
        } else if (now - stall_start >= std::chrono::seconds(5)) {
          throw std::runtime_error(std::string("send failed: ") + std::strerror(errno) +
                                   " for 5 s without progress");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(backoff_us));
        backoff_us = std::min(2 * backoff_us, 100000L);
        continue;
      }
      throw std::runtime_error(std::string("send failed: ") + std::strerror(errno));
    }
    stalled = false;
    backoff_us = 1000;
    size_t left = static_cast<size_t>(w);
    const size_t th = std::min(left, hdr.size() - sent_h);
    sent_h += th;
    left -= th;
    sent_p += left;
  }
  return hdr.size() + n;
}

void recv_exact(int fd, char* dst, size_t n) {
  size_t got = 0;
  while (got < n) {
    const ssize_t r = recv(fd, dst + got, n - got, 0);
    if (r == 0) throw std::runtime_error("peer closed");
    if (r < 0) {
      if (errno == EINTR) continue;
      throw std::runtime_error(std::string("recv failed: ") + std::strerror(errno));
    }
    got += static_cast<size_t>(r);
  }
}

// -> (type, codec, step, mb, chunk, shape, frag_idx, frag_cnt, payload)
py::tuple recv_frame(int fd, uint64_t max_payload) {
  Header h{};
  std::vector<uint32_t> shape;
  std::string payload;
  {
    py::gil_scoped_release nogil;
    recv_exact(fd, reinterpret_cast<char*>(&h), sizeof(h));
    if (h.magic != kMagic) throw std::runtime_error("bad frame magic");
    if (h.type > 7) throw std::runtime_error("unknown frame type");
    shape.resize(h.ndim);
    if (h.ndim) recv_exact(fd, reinterpret_cast<char*>(shape.data()), 4 * h.ndim);
    uint64_t n = 0;
    recv_exact(fd, reinterpret_cast<char*>(&n), 8);
    if (n > max_payload) throw std::runtime_error("frame payload exceeds the limit");
    payload.resize(n);
    if (n) recv_exact(fd, &payload[0], n);
  }
  return py::make_tuple(static_cast<int>(h.type), static_cast<int>(h.codec), h.step, h.mb,
                        static_cast<int>(h.chunk), shape, static_cast<int>(h.frag_idx),
                        static_cast<int>(h.frag_cnt), py::bytes(payload));
}

}  // namespace

PYBIND11_MODULE(_wire, m) {
  m.doc() = "Native codecs and frame I/O of the TCP data plane";
  m.def("planes_encode", &planes_encode, py::arg("data"), py::arg("esz"), py::arg("dtype_id"),
        py::arg("level") = 1);
  m.def("planes_decode", &planes_decode, py::arg("payload"), py::arg("esz"));
  m.def("pair_encode", &pair_encode, py::arg("a"), py::arg("b"), py::arg("b_esz"),
        py::arg("dtype_id"), py::arg("level") = 1);
  m.def("pair_decode", &pair_decode, py::arg("payload"), py::arg("b_esz"));
  m.def("fp8_planes_encode", &fp8_planes_encode, py::arg("codes"), py::arg("level") = 1);
  m.def("fp8_planes_decode", &fp8_planes_decode);
  m.def("f32_planes_encode", &f32_planes_encode, py::arg("data"), py::arg("level") = 1);
  m.def("f32_planes_decode", &f32_planes_decode);
  m.def("pack_header", &pack_header);
  m.def("send_frame", &send_frame);
  m.def("recv_frame", &recv_frame);
  m.def("set_threads", [](int n) { g_threads = n; }, "codec threads (0 = all cores)");
  m.attr("MAGIC") = kMagic;
}
