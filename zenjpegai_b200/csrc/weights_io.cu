// Checkpoint readers (host code only): PyTorch `.pth` files (an uncompressed ZIP holding a
// pickled state dict and one member per tensor storage) and the crate's packed containers
// (`ZJM1` checkpoints, `ZJB1` / `ZJB2` bundles), exposing the tensors by name the way
// src/weights/mod.rs `Checkpoint` does, and the floating-point ones as `zjai_param`s for
// zjai_net_create. Behaviour follows src/weights/{mod,zip,pickle,packed,dtype}.rs: the same
// accepted storage classes and dtype codes, tensors at the top level of the root dict, nested
// dicts flattened to dotted names up to three levels (their tensors and numeric lists), integer
// entries, strided views gathered into contiguous bytes, f16 tensors upcast for the f32 view.
// Every read is bounds-checked: a malformed file fails with ZJAI_MODEL, never reads outside
// the buffer. The pickle interpreter only builds data (no code runs): a global is a name pair,
// and only torch's tensor / parameter rebuilds and OrderedDict are given meaning.
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "api_common.h"

namespace zjai {
namespace wio {

// Element types; the numbering is the ZJM1 dtype code (src/weights/packed.rs:61-75).
enum DType : int { F64 = 0, F32 = 1, F16 = 2, I64 = 3, I32 = 4, I16 = 5, I8 = 6, U8 = 7, BOOL = 8 };

int dtype_size(int d) {
  switch (d) {
    case F64:
    case I64: return 8;
    case F32:
    case I32: return 4;
    case F16:
    case I16: return 2;
    default: return 1;
  }
}

// torch storage class -> element type (src/weights/dtype.rs:35-48)
bool dtype_of_storage(const std::string& cls, int* d) {
  static const std::pair<const char*, int> tab[] = {
      {"DoubleStorage", F64}, {"FloatStorage", F32}, {"HalfStorage", F16},
      {"LongStorage", I64},   {"IntStorage", I32},   {"ShortStorage", I16},
      {"CharStorage", I8},    {"ByteStorage", U8},   {"BoolStorage", BOOL}};
  for (auto& e : tab)
    if (cls == e.first) {
      *d = e.second;
      return true;
    }
  return false;
}

constexpr uint32_t kMaxEntries = 1u << 20;  // table sizes accepted (hostile-input bound)
constexpr int kMaxRank = 8;
// Largest dimension, stride, storage offset and element count accepted: with rank <= 8 every
// product and index sum below stays far inside 128 bits, so no bound check can be defeated by
// wrap-around.
constexpr uint64_t kMaxExtent = (uint64_t)1 << 40;

// Bounds-checked little-endian cursor over [p, p + n).
struct Cursor {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  Cursor(const uint8_t* d, size_t len) : p(d), n(len) {}
  const uint8_t* take(size_t k) {
    if (!ok || k > n - pos) {
      ok = false;
      return nullptr;
    }
    const uint8_t* r = p + pos;
    pos += k;
    return r;
  }
  uint64_t le(int bytes) {
    const uint8_t* b = take((size_t)bytes);
    uint64_t v = 0;
    if (b)
      for (int i = bytes - 1; i >= 0; --i) v = (v << 8) | b[i];
    return v;
  }
  uint8_t u8() { return (uint8_t)le(1); }
  uint16_t u16() { return (uint16_t)le(2); }
  uint32_t u32() { return (uint32_t)le(4); }
  uint64_t u64() { return le(8); }
};

// Well-formed UTF-8 (names, paths and pickle text must be; the crate rejects the rest)
bool utf8_ok(const uint8_t* p, size_t n) {
  for (size_t i = 0; i < n;) {
    const uint8_t c = p[i];
    size_t k;
    uint32_t cp;
    if (c < 0x80) {
      ++i;
      continue;
    } else if ((c & 0xE0) == 0xC0) {
      k = 1;
      cp = c & 0x1F;
    } else if ((c & 0xF0) == 0xE0) {
      k = 2;
      cp = c & 0x0F;
    } else if ((c & 0xF8) == 0xF0) {
      k = 3;
      cp = c & 0x07;
    } else {
      return false;
    }
    if (k > n - i - 1) return false;
    for (size_t j = 1; j <= k; ++j) {
      if ((p[i + j] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + j] & 0x3F);
    }
    if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) ||
        cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))
      return false;
    i += k + 1;
  }
  return true;
}

uint64_t rd_le(const uint8_t* b, int bytes) {
  uint64_t v = 0;
  for (int i = bytes - 1; i >= 0; --i) v = (v << 8) | b[i];
  return v;
}

// ---- ZIP (stored members only, as torch.save writes them; ZIP64 records honoured) ---------

struct ZipMember {
  size_t off, len;  // data span in the archive
};

int zip_members(const uint8_t* f, size_t n, std::map<std::string, ZipMember>* out) {
  // end of central directory: the last "PK\5\6" with room for its 22 bytes
  if (n < 22) return fail(ZJAI_MODEL, "zip: file too short");
  size_t eocd = SIZE_MAX;
  const size_t lo = n > 22 + 65535 ? n - 22 - 65535 : 0;
  for (size_t i = n - 22 + 1; i-- > lo;)
    if (rd_le(f + i, 4) == 0x06054b50u) {
      eocd = i;
      break;
    }
  if (eocd == SIZE_MAX) return fail(ZJAI_MODEL, "zip: no end-of-central-directory record");
  uint64_t count = rd_le(f + eocd + 10, 2), cd_size = rd_le(f + eocd + 12, 4),
           cd_off = rd_le(f + eocd + 16, 4);
  if (count == 0xFFFF || cd_off == 0xFFFFFFFFu || cd_size == 0xFFFFFFFFu) {
    // ZIP64: the locator sits right before the record and points at the ZIP64 record
    if (eocd < 20 || rd_le(f + eocd - 20, 4) != 0x07064b50u)
      return fail(ZJAI_MODEL, "zip: ZIP64 locator missing");
    const uint64_t z = rd_le(f + eocd - 20 + 8, 8);
    if (z > n || n - z < 56 || rd_le(f + z, 4) != 0x06064b50u)
      return fail(ZJAI_MODEL, "zip: ZIP64 end record invalid");
    count = rd_le(f + z + 32, 8);
    cd_size = rd_le(f + z + 40, 8);
    cd_off = rd_le(f + z + 48, 8);
  }
  if (count > kMaxEntries) return fail(ZJAI_LIMIT_EXCEEDED, "zip: too many members");
  if (cd_off > n || cd_size > n - cd_off) return fail(ZJAI_MODEL, "zip: central directory out of range");
  Cursor c(f + cd_off, (size_t)cd_size);
  for (uint64_t e = 0; e < count; ++e) {
    if (c.u32() != 0x02014b50u) return fail(ZJAI_MODEL, "zip: bad central directory entry");
    c.take(6);
    const uint16_t method = c.u16();
    c.take(8);
    uint64_t csize = c.u32(), usize = c.u32();
    const uint16_t nlen = c.u16(), xlen = c.u16(), clen = c.u16();
    c.take(8);
    uint64_t lho = c.u32();
    const uint8_t* name = c.take(nlen);
    const uint8_t* extra = c.take(xlen);
    c.take(clen);
    if (!c.ok) return fail(ZJAI_MODEL, "zip: truncated central directory");
    // ZIP64 extended information: the 64-bit values of the fields saturated above, in order
    for (size_t x = 0; x + 4 <= xlen;) {
      const uint16_t id = (uint16_t)rd_le(extra + x, 2), sz = (uint16_t)rd_le(extra + x + 2, 2);
      if (x + 4 + sz > xlen) break;
      if (id == 0x0001) {
        size_t q = x + 4;
        auto next = [&](uint64_t* v) {
          if (*v == 0xFFFFFFFFu && q + 8 <= x + 4 + sz) {
            *v = rd_le(extra + q, 8);
            q += 8;
          }
        };
        next(&usize);
        next(&csize);
        next(&lho);
      }
      x += 4 + sz;
    }
    if (method != 0) return fail(ZJAI_MODEL, "zip: compressed member (only stored members are read)");
    if (csize != usize) return fail(ZJAI_MODEL, "zip: stored member with differing sizes");
    if (lho > n || n - lho < 30 || rd_le(f + lho, 4) != 0x04034b50u)
      return fail(ZJAI_MODEL, "zip: bad local header");
    const uint64_t data = lho + 30 + rd_le(f + lho + 26, 2) + rd_le(f + lho + 28, 2);
    if (data > n || usize > n - data) return fail(ZJAI_MODEL, "zip: member data out of range");
    (*out)[std::string(reinterpret_cast<const char*>(name), nlen)] = {(size_t)data, (size_t)usize};
  }
  return ZJAI_OK;
}

// ---- pickle (the opcodes of protocols 0-4 that state dicts use; data only) ------------------

struct TRef {
  std::string key;  // storage: archive member <prefix>data/<key>
  int dtype = F32;
  uint64_t offset = 0;  // in elements
  std::vector<uint64_t> shape, stride;
};

struct Value;
using VP = std::shared_ptr<Value>;
struct Value {
  enum Kind { NONE, BOOL, INT, FLOAT, STR, BYTES, TUPLE, LIST, DICT, GLOBAL, STORAGE, TENSOR, OBJECT };
  Kind k = NONE;
  int64_t i = 0;
  double f = 0.0;
  std::string s, s2;  // STR / BYTES text; GLOBAL module, name
  std::vector<VP> items;
  std::vector<std::pair<VP, VP>> dict;
  TRef t;
};

VP mk(Value::Kind k) {
  VP v = std::make_shared<Value>();
  v->k = k;
  return v;
}

constexpr size_t kMaxStack = 1u << 20, kMaxMemo = 1u << 22;

bool as_u64(const VP& v, uint64_t* out) {
  if (!v || v->k != Value::INT || v->i < 0) return false;
  *out = (uint64_t)v->i;
  return true;
}
bool as_u64_list(const VP& v, std::vector<uint64_t>* out) {
  if (!v || (v->k != Value::TUPLE && v->k != Value::LIST)) return false;
  out->clear();
  for (auto& x : v->items) {
    uint64_t u;
    if (!as_u64(x, &u)) return false;
    out->push_back(u);
  }
  return true;
}

// callable(args) for the callables the interpreter knows (src/weights/pickle.rs:150-177)
VP reduce(const VP& fn, const VP& args) {
  if (fn->k == Value::GLOBAL && args->k == Value::TUPLE) {
    const std::string& m = fn->s;
    const std::string& n = fn->s2;
    const auto& a = args->items;
    if (m == "collections" && n == "OrderedDict" && a.empty()) return mk(Value::DICT);
    if (m == "torch._utils" && n == "_rebuild_tensor_v2" && a.size() >= 4 &&
        a[0]->k == Value::STORAGE) {
      VP t = mk(Value::TENSOR);
      t->t.key = a[0]->s;
      t->t.dtype = (int)a[0]->i;
      if (as_u64(a[1], &t->t.offset) && as_u64_list(a[2], &t->t.shape) &&
          as_u64_list(a[3], &t->t.stride))
        return t;
    }
    if (m == "torch._utils" && n == "_rebuild_parameter" && !a.empty()) return a[0];
  }
  VP o = mk(Value::OBJECT);
  o->items = {fn, args};
  return o;
}

// persistent id ('storage', <StorageClass>, key, location, numel) -> a storage reference
int persistent(const VP& pid, VP* out) {
  if (pid->k != Value::TUPLE || pid->items.size() < 3 || pid->items[0]->k != Value::STR ||
      pid->items[0]->s != "storage" || pid->items[1]->k != Value::GLOBAL ||
      pid->items[2]->k != Value::STR)
    return fail(ZJAI_MODEL, "pickle: unrecognised persistent id");
  int d;
  if (!dtype_of_storage(pid->items[1]->s2, &d))
    return fail(ZJAI_MODEL, "pickle: unsupported storage class `" + pid->items[1]->s2 + "`");
  VP v = mk(Value::STORAGE);
  v->s = pid->items[2]->s;
  v->i = d;
  *out = v;
  return ZJAI_OK;
}

int unpickle(const uint8_t* data, size_t len, VP* root) {
  Cursor r(data, len);
  std::vector<VP> st;
  std::vector<size_t> marks;
  std::vector<VP> memo;
  auto bad = [](const char* m) { return fail(ZJAI_MODEL, std::string("pickle: ") + m); };
  auto pop = [&](VP* v) {
    if (st.empty() || (!marks.empty() && marks.back() == st.size())) return false;
    *v = st.back();
    st.pop_back();
    return true;
  };
  auto pop_mark = [&](std::vector<VP>* items) {
    if (marks.empty() || marks.back() > st.size()) return false;
    items->assign(st.begin() + (long)marks.back(), st.end());
    st.resize(marks.back());
    marks.pop_back();
    return true;
  };
  auto line = [&](std::string* out) {
    out->clear();
    for (;;) {
      const uint8_t* b = r.take(1);
      if (!b) return false;
      if (*b == '\n') return true;
      out->push_back((char)*b);
    }
  };
  auto str = [&](Value::Kind k, uint64_t n) {
    const uint8_t* b = r.take((size_t)n);
    if (!b || (k == Value::STR && !utf8_ok(b, (size_t)n))) return false;
    VP v = mk(k);
    v->s.assign(reinterpret_cast<const char*>(b), (size_t)n);
    st.push_back(v);
    return true;
  };
  auto memo_put = [&](uint64_t idx) {
    if (st.empty() || idx >= kMaxMemo) return false;
    if (memo.size() <= idx) memo.resize(idx + 1);
    memo[idx] = st.back();
    return true;
  };
  auto memo_get = [&](uint64_t idx) {
    if (idx >= memo.size() || !memo[idx]) return false;
    st.push_back(memo[idx]);
    return true;
  };
  for (;;) {
    if (st.size() > kMaxStack) return fail(ZJAI_LIMIT_EXCEEDED, "pickle: stack too deep");
    const uint8_t* ob = r.take(1);
    if (!ob) return bad("truncated (no STOP)");
    VP a, b, c;
    std::vector<VP> items;
    switch (*ob) {
      case 0x80: r.take(1); break;  // PROTO
      case 0x95: r.take(8); break;  // FRAME
      case '.':                    // STOP
        if (!pop(&a)) return bad("STOP on an empty stack");
        *root = a;
        return ZJAI_OK;
      case '(': marks.push_back(st.size()); break;
      case 'N': st.push_back(mk(Value::NONE)); break;
      case 0x88:
      case 0x89:
        a = mk(Value::BOOL);
        a->i = *ob == 0x88;
        st.push_back(a);
        break;
      case 'J': a = mk(Value::INT); a->i = (int32_t)r.u32(); st.push_back(a); break;
      case 'K': a = mk(Value::INT); a->i = r.u8(); st.push_back(a); break;
      case 'M': a = mk(Value::INT); a->i = r.u16(); st.push_back(a); break;
      case 0x8a:  // LONG1: n little-endian two's-complement bytes
      case 0x8b: {
        const uint64_t n = *ob == 0x8a ? r.u8() : r.u32();
        if (n > 8) return bad("integer wider than 64 bits");
        const uint8_t* d = r.take((size_t)n);
        if (!d) return bad("truncated LONG");
        uint64_t u = n ? rd_le(d, (int)n) : 0;
        if (n && n < 8 && (d[n - 1] & 0x80)) u |= ~0ull << (8 * n);  // sign-extend
        a = mk(Value::INT);
        a->i = (int64_t)u;
        st.push_back(a);
        break;
      }
      case 'I': {  // INT as text ("01" / "00" are True / False)
        std::string t;
        if (!line(&t)) return bad("truncated INT");
        a = mk(Value::INT);
        a->i = t == "01" ? 1 : t == "00" ? 0 : std::strtoll(t.c_str(), nullptr, 10);
        st.push_back(a);
        break;
      }
      case 'G': {  // BINFLOAT, big-endian
        const uint8_t* d = r.take(8);
        if (!d) return bad("truncated BINFLOAT");
        uint64_t u = 0;
        for (int k = 0; k < 8; ++k) u = (u << 8) | d[k];
        a = mk(Value::FLOAT);
        std::memcpy(&a->f, &u, 8);
        st.push_back(a);
        break;
      }
      case 'X': if (!str(Value::STR, r.u32())) return bad("truncated string"); break;
      case 0x8c: if (!str(Value::STR, r.u8())) return bad("truncated string"); break;
      case 0x8d: if (!str(Value::STR, r.u64())) return bad("truncated string"); break;
      case 'T': if (!str(Value::STR, r.u32())) return bad("truncated string"); break;
      case 'U': if (!str(Value::STR, r.u8())) return bad("truncated string"); break;
      case 'B': if (!str(Value::BYTES, r.u32())) return bad("truncated bytes"); break;
      case 'C': if (!str(Value::BYTES, r.u8())) return bad("truncated bytes"); break;
      case 0x8e: if (!str(Value::BYTES, r.u64())) return bad("truncated bytes"); break;
      case 'c': {  // GLOBAL module\nname\n
        a = mk(Value::GLOBAL);
        if (!line(&a->s) || !line(&a->s2)) return bad("truncated GLOBAL");
        st.push_back(a);
        break;
      }
      case 0x93:  // STACK_GLOBAL
        if (!pop(&b) || !pop(&a) || a->k != Value::STR || b->k != Value::STR)
          return bad("STACK_GLOBAL operands are not strings");
        c = mk(Value::GLOBAL);
        c->s = a->s;
        c->s2 = b->s;
        st.push_back(c);
        break;
      case ')': st.push_back(mk(Value::TUPLE)); break;
      case 't':
        if (!pop_mark(&items)) return bad("TUPLE without a mark");
        a = mk(Value::TUPLE);
        a->items = items;
        st.push_back(a);
        break;
      case 0x85:
      case 0x86:
      case 0x87: {
        const int n = *ob - 0x84;
        a = mk(Value::TUPLE);
        a->items.resize(n);
        for (int k = n - 1; k >= 0; --k)
          if (!pop(&a->items[k])) return bad("stack underflow");
        st.push_back(a);
        break;
      }
      case ']': st.push_back(mk(Value::LIST)); break;
      case 'l':
        if (!pop_mark(&items)) return bad("LIST without a mark");
        a = mk(Value::LIST);
        a->items = items;
        st.push_back(a);
        break;
      case 'a':
        if (!pop(&b) || st.empty() || st.back()->k != Value::LIST) return bad("APPEND target");
        st.back()->items.push_back(b);
        break;
      case 'e':
        if (!pop_mark(&items) || st.empty() || st.back()->k != Value::LIST)
          return bad("APPENDS target");
        for (auto& x : items) st.back()->items.push_back(x);
        break;
      case '}': st.push_back(mk(Value::DICT)); break;
      case 'd':
        if (!pop_mark(&items) || items.size() % 2) return bad("DICT operands");
        a = mk(Value::DICT);
        for (size_t k = 0; k < items.size(); k += 2) a->dict.push_back({items[k], items[k + 1]});
        st.push_back(a);
        break;
      case 's':
        if (!pop(&c) || !pop(&b) || st.empty()) return bad("SETITEM operands");
        if (st.back()->k == Value::DICT) st.back()->dict.push_back({b, c});
        else if (st.back()->k != Value::OBJECT) return bad("SETITEM target is not a dict");
        break;
      case 'u':
        if (!pop_mark(&items) || items.size() % 2 || st.empty()) return bad("SETITEMS operands");
        if (st.back()->k == Value::DICT)
          for (size_t k = 0; k < items.size(); k += 2) st.back()->dict.push_back({items[k], items[k + 1]});
        else if (st.back()->k != Value::OBJECT) return bad("SETITEMS target is not a dict");
        break;
      case 'R':
      case 0x81:  // REDUCE / NEWOBJ
        if (!pop(&b) || !pop(&a)) return bad("REDUCE operands");
        st.push_back(reduce(a, b));
        break;
      case 'b':  // BUILD: the state of an object; the interpreter keeps no object state
        if (!pop(&a) || st.empty()) return bad("BUILD operands");
        break;
      case 'Q': {  // BINPERSID
        if (!pop(&a)) return bad("BINPERSID operand");
        VP v;
        ZJAI_TRY(persistent(a, &v));
        st.push_back(v);
        break;
      }
      case 'q': if (!memo_put(r.u8())) return bad("BINPUT"); break;
      case 'r': if (!memo_put(r.u32())) return bad("LONG_BINPUT"); break;
      case 0x94: if (!memo_put(memo.size())) return bad("MEMOIZE"); break;
      case 'h': if (!memo_get(r.u8())) return bad("BINGET of an unset slot"); break;
      case 'j': if (!memo_get(r.u32())) return bad("LONG_BINGET of an unset slot"); break;
      case '0': if (!pop(&a)) return bad("POP on an empty stack"); break;
      case '2':
        if (st.empty()) return bad("DUP on an empty stack");
        st.push_back(st.back());
        break;
      case '1':
        if (!pop_mark(&items)) return bad("POP_MARK without a mark");
        break;
      default: {
        char m[64];
        snprintf(m, sizeof m, "unsupported opcode 0x%02x", *ob);
        return bad(m);
      }
    }
    if (!r.ok) return bad("truncated");
  }
}

// ---- checkpoints ------------------------------------------------------------------------

struct Ckpt {
  std::vector<uint8_t> file;  // the file's bytes (owned)
  bool packed = false;        // ZJM1: every tensor's storage is the file itself
  std::map<std::string, ZipMember> members;
  std::string prefix;  // "<archive>/" of the .pth members
  std::vector<std::pair<std::string, TRef>> tensors;
  std::vector<std::pair<std::string, int64_t>> ints;
  std::vector<std::pair<std::string, std::vector<double>>> lists;
  // the floating-point tensors as f32 parameters (built on first request)
  bool params_built = false;
  std::vector<std::vector<float>> f32;
  std::vector<zjai_param> params;
};

// Nested dicts of the root (`clip_thres` tables, optimizer state): their tensors and numeric
// lists under dotted names, three levels deep at most (src/weights/mod.rs:83-125).
void flatten_nested(const std::string& prefix, const std::vector<std::pair<VP, VP>>& items,
                    int depth, Ckpt* ck) {
  if (depth >= 3) return;
  for (auto& kv : items) {
    if (kv.first->k != Value::STR) continue;
    const std::string name = prefix + "." + kv.first->s;
    const VP& v = kv.second;
    if (v->k == Value::TENSOR) {
      ck->tensors.push_back({name, v->t});
    } else if (v->k == Value::DICT) {
      flatten_nested(name, v->dict, depth + 1, ck);
    } else if (v->k == Value::LIST) {
      std::vector<double> xs;
      bool num = true;
      for (auto& x : v->items) {
        if (x->k == Value::FLOAT) xs.push_back(x->f);
        else if (x->k == Value::INT) xs.push_back((double)x->i);
        else num = false;
      }
      if (num) ck->lists.push_back({name, xs});
    }
  }
}

int parse_pth(Ckpt* ck) {
  ZJAI_TRY(zip_members(ck->file.data(), ck->file.size(), &ck->members));
  const ZipMember* pkl = nullptr;
  for (auto& m : ck->members) {
    const std::string& n = m.first;
    if (n == "data.pkl" || (n.size() > 9 && n.compare(n.size() - 9, 9, "/data.pkl") == 0)) {
      pkl = &m.second;
      ck->prefix = n.substr(0, n.size() - 8);
      break;
    }
  }
  if (!pkl) return fail(ZJAI_MODEL, "checkpoint has no data.pkl");
  VP root;
  ZJAI_TRY(unpickle(ck->file.data() + pkl->off, pkl->len, &root));
  if (root->k != Value::DICT) return fail(ZJAI_MODEL, "checkpoint root is not a state dict");
  for (auto& kv : root->dict) {
    if (kv.first->k != Value::STR) continue;
    const VP& v = kv.second;
    if (v->k == Value::TENSOR) ck->tensors.push_back({kv.first->s, v->t});
    else if (v->k == Value::INT) ck->ints.push_back({kv.first->s, v->i});
    else if (v->k == Value::DICT) flatten_nested(kv.first->s, v->dict, 0, ck);
  }
  return ZJAI_OK;
}

// ZJM1 tables (src/weights/packed.rs:8-21, 149-197)
int parse_zjm(Ckpt* ck) {
  Cursor r(ck->file.data(), ck->file.size());
  r.take(4);
  if (r.u32() != 1) return fail(ZJAI_MODEL, "packed model: unsupported version");
  const uint32_t nt = r.u32(), ni = r.u32();
  if (!r.ok) return fail(ZJAI_MODEL, "packed model: truncated table");
  if (nt > kMaxEntries || ni > kMaxEntries)
    return fail(ZJAI_LIMIT_EXCEEDED, "packed model: too many entries");
  auto str = [&](std::string* out) {
    const uint16_t n = r.u16();
    const uint8_t* b = r.take(n);
    if (b) out->assign(reinterpret_cast<const char*>(b), n);
    return r.ok && (!b || utf8_ok(b, n));
  };
  for (uint32_t i = 0; i < nt; ++i) {
    std::string name;
    if (!str(&name)) return fail(ZJAI_MODEL, "packed model: truncated table or name not UTF-8");
    TRef t;
    t.dtype = r.u8();
    const int rank = r.u8();
    if (t.dtype > BOOL) return fail(ZJAI_MODEL, "packed model: unknown dtype code");
    if (rank > kMaxRank) return fail(ZJAI_MODEL, "packed model: tensor rank above 8");
    for (int k = 0; k < rank; ++k) t.shape.push_back(r.u64());
    const uint64_t off = r.u64(), len = r.u64();
    if (!r.ok) return fail(ZJAI_MODEL, "packed model: truncated table");
    const uint64_t es = (uint64_t)dtype_size(t.dtype);
    unsigned __int128 numel = es;
    bool big = false;
    for (uint64_t d : t.shape) {
      big = big || d > kMaxExtent;
      numel *= d;
      big = big || numel > (unsigned __int128)kMaxExtent;
      if (big) break;
    }
    if (big) return fail(ZJAI_LIMIT_EXCEEDED, "packed model: tensor `" + name + "` too large");
    if (numel != len || off % 64 || off > ck->file.size() || len > ck->file.size() - off)
      return fail(ZJAI_MODEL, "packed model: tensor `" + name + "` has an invalid extent");
    t.stride.assign(rank, 1);
    for (int ax = rank - 2; ax >= 0; --ax) t.stride[ax] = t.stride[ax + 1] * t.shape[ax + 1];
    t.offset = off / es;
    ck->tensors.push_back({name, t});
  }
  for (uint32_t i = 0; i < ni; ++i) {
    std::string name;
    if (!str(&name)) return fail(ZJAI_MODEL, "packed model: truncated table or name not UTF-8");
    const int64_t v = (int64_t)r.u64();
    if (!r.ok) return fail(ZJAI_MODEL, "packed model: truncated table");
    ck->ints.push_back({name, v});
  }
  ck->packed = true;
  return ZJAI_OK;
}

// Contiguous row-major bytes of tensor t (a strided view is gathered element by element),
// every index checked against its storage (src/weights/mod.rs:245-330).
int tensor_bytes(const Ckpt* ck, const std::string& name, const TRef& t, std::vector<uint8_t>* out) {
  const uint8_t* st;
  size_t st_len;
  if (ck->packed) {
    st = ck->file.data();
    st_len = ck->file.size();
  } else {
    auto it = ck->members.find(ck->prefix + "data/" + t.key);
    if (it == ck->members.end())
      return fail(ZJAI_MODEL, "tensor `" + name + "`: storage `" + t.key + "` missing");
    st = ck->file.data() + it->second.off;
    st_len = it->second.len;
  }
  if (t.shape.size() != t.stride.size())
    return fail(ZJAI_MODEL, "tensor `" + name + "`: shape/stride rank mismatch");
  const size_t es = (size_t)dtype_size(t.dtype), elems = st_len / es;
  if (t.shape.size() > (size_t)kMaxRank || t.offset > kMaxExtent)
    return fail(ZJAI_LIMIT_EXCEEDED, "tensor `" + name + "`: rank or offset too large");
  unsigned __int128 numel = 1, last = t.offset;  // highest element index the view touches
  bool empty = false;
  for (size_t a = 0; a < t.shape.size(); ++a) {
    if (t.shape[a] > kMaxExtent || t.stride[a] > kMaxExtent)
      return fail(ZJAI_LIMIT_EXCEEDED, "tensor `" + name + "`: extent or stride too large");
    numel *= t.shape[a];
    if (numel * es > kMaxExtent) return fail(ZJAI_LIMIT_EXCEEDED, "tensor too large");
    if (t.shape[a] == 0) empty = true;
    else last += (unsigned __int128)(t.shape[a] - 1) * t.stride[a];
  }
  out->assign((size_t)(numel * es), 0);
  if (empty) return ZJAI_OK;
  if (last >= elems) return fail(ZJAI_MODEL, "tensor `" + name + "` exceeds its storage");
  bool contiguous = true;
  uint64_t expect = 1;
  for (size_t a = t.shape.size(); a-- > 0;) {
    if (t.shape[a] != 1 && t.stride[a] != expect) contiguous = false;
    expect *= t.shape[a];
  }
  if (contiguous) {
    std::memcpy(out->data(), st + t.offset * es, out->size());
    return ZJAI_OK;
  }
  const size_t rank = t.shape.size();
  std::vector<uint64_t> idx(rank, 0);
  for (size_t e = 0; e < (size_t)numel; ++e) {
    uint64_t src = t.offset;
    for (size_t a = 0; a < rank; ++a) src += idx[a] * t.stride[a];
    std::memcpy(out->data() + e * es, st + src * es, es);
    for (size_t a = rank; a-- > 0;) {
      if (++idx[a] < t.shape[a]) break;
      idx[a] = 0;
    }
  }
  return ZJAI_OK;
}

// IEEE binary16 -> binary32, exact
float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {  // subnormal: m * 2^-24, normalised
      int sh = 0;
      uint32_t mm = m;
      while (!(mm & 1024u)) {
        mm <<= 1;
        ++sh;
      }
      bits = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | ((mm & 1023u) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7F800000u | (m << 13);
  } else {
    bits = sign | ((e - 15 + 127) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

int build_params(Ckpt* ck) {
  if (ck->params_built) return ZJAI_OK;
  ck->f32.clear();
  ck->params.clear();
  for (auto& nt : ck->tensors) {
    const TRef& t = nt.second;
    if ((t.dtype != F32 && t.dtype != F16) || t.shape.size() > 4) continue;
    std::vector<uint8_t> raw;
    ZJAI_TRY(tensor_bytes(ck, nt.first, t, &raw));
    std::vector<float> v(raw.size() / (size_t)dtype_size(t.dtype));
    if (t.dtype == F32) {
      std::memcpy(v.data(), raw.data(), raw.size());
    } else {
      for (size_t i = 0; i < v.size(); ++i)
        v[i] = half_to_float((uint16_t)(raw[2 * i] | raw[2 * i + 1] << 8));
    }
    ck->f32.push_back(std::move(v));
  }
  size_t k = 0;
  for (auto& nt : ck->tensors) {
    const TRef& t = nt.second;
    if ((t.dtype != F32 && t.dtype != F16) || t.shape.size() > 4) continue;
    zjai_param p;
    std::memset(&p, 0, sizeof p);
    p.name = nt.first.c_str();
    p.ndim = (int)t.shape.size();
    for (int a = 0; a < p.ndim; ++a) p.shape[a] = (int64_t)t.shape[a];
    p.data = ck->f32[k++].data();
    ck->params.push_back(p);
  }
  ck->params_built = true;
  return ZJAI_OK;
}

// ZJB1 / ZJB2 bundle (src/weights/packed.rs:23-43, 292-330)
struct Bundle {
  std::vector<uint8_t> file;
  bool f16 = false;
  std::string notice;
  std::vector<std::pair<std::string, ZipMember>> files;
};

int parse_bundle(Bundle* b) {
  Cursor r(b->file.data(), b->file.size());
  r.take(4);
  if (r.u32() != 1) return fail(ZJAI_MODEL, "bundle: unsupported version");
  const uint32_t nf = r.u32(), nn = r.u32();
  if (!r.ok) return fail(ZJAI_MODEL, "bundle: truncated table");
  if (nf > kMaxEntries) return fail(ZJAI_LIMIT_EXCEEDED, "bundle: too many files");
  const uint8_t* nb = r.take(nn);
  if (!nb) return fail(ZJAI_MODEL, "bundle: truncated notice");
  if (!utf8_ok(nb, nn)) return fail(ZJAI_MODEL, "bundle: notice is not UTF-8");
  b->notice.assign(reinterpret_cast<const char*>(nb), nn);
  for (uint32_t i = 0; i < nf; ++i) {
    const uint16_t n = r.u16();
    const uint8_t* p = r.take(n);
    const uint64_t off = r.u64(), len = r.u64();
    if (!r.ok) return fail(ZJAI_MODEL, "bundle: truncated table");
    if (!utf8_ok(p, n)) return fail(ZJAI_MODEL, "bundle: path is not UTF-8");
    if (off % 64 || off > b->file.size() || len > b->file.size() - off)
      return fail(ZJAI_MODEL, "bundle: file with an invalid extent");
    b->files.push_back({std::string(reinterpret_cast<const char*>(p), n),
                        {(size_t)off, (size_t)len}});
  }
  return ZJAI_OK;
}

}  // namespace wio
}  // namespace zjai

// ---- C ABI -------------------------------------------------------------------------------

struct zjai_ckpt : zjai::wio::Ckpt {};
struct zjai_bundle : zjai::wio::Bundle {};

using namespace zjai;

int zjai_ckpt_open(const void* data, size_t len, zjai_ckpt** out) {
  if (!out) return fail(ZJAI_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  if (!data && len) return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: null data");
  try {
    std::unique_ptr<zjai_ckpt> ck(new zjai_ckpt());
    const uint8_t* p = static_cast<const uint8_t*>(data);
    ck->file.assign(p, p + len);
    if (len >= 4 && std::memcmp(p, "ZJM1", 4) == 0) ZJAI_TRY(wio::parse_zjm(ck.get()));
    else ZJAI_TRY(wio::parse_pth(ck.get()));
    *out = ck.release();
    return ZJAI_OK;
  } catch (const std::bad_alloc&) {
    return fail(ZJAI_LIMIT_EXCEEDED, "checkpoint: out of host memory");
  }
}

int zjai_ckpt_close(zjai_ckpt* ck) {
  delete ck;
  return ZJAI_OK;
}

int zjai_ckpt_count(const zjai_ckpt* ck, int* ntensors, int* nints, int* nlists) {
  if (!ck) return fail(ZJAI_INVALID_ARGUMENT, "null checkpoint");
  if (ntensors) *ntensors = (int)ck->tensors.size();
  if (nints) *nints = (int)ck->ints.size();
  if (nlists) *nlists = (int)ck->lists.size();
  return ZJAI_OK;
}

int zjai_ckpt_tensor(const zjai_ckpt* ck, int i, const char** name, int* dtype, int* ndim,
                     int64_t* shape) {
  if (!ck || i < 0 || i >= (int)ck->tensors.size())
    return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: tensor index out of range");
  const wio::TRef& t = ck->tensors[i].second;
  if (name) *name = ck->tensors[i].first.c_str();
  if (dtype) *dtype = t.dtype;
  if (ndim) *ndim = (int)t.shape.size();
  if (shape)
    for (size_t a = 0; a < t.shape.size(); ++a) shape[a] = (int64_t)t.shape[a];
  return ZJAI_OK;
}

int zjai_ckpt_find(const zjai_ckpt* ck, const char* name, int* index) {
  if (!ck || !name || !index) return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: bad arguments");
  for (size_t i = 0; i < ck->tensors.size(); ++i)
    if (ck->tensors[i].first == name) {
      *index = (int)i;
      return ZJAI_OK;
    }
  return fail(ZJAI_MODEL, std::string("tensor `") + name + "` not found");
}

int zjai_ckpt_read(const zjai_ckpt* ck, int i, void* dst, size_t capacity) {
  if (!ck || i < 0 || i >= (int)ck->tensors.size())
    return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: tensor index out of range");
  try {
    std::vector<uint8_t> raw;
    ZJAI_TRY(wio::tensor_bytes(ck, ck->tensors[i].first, ck->tensors[i].second, &raw));
    if (raw.size() > capacity || (!dst && !raw.empty()))
      return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: destination smaller than the tensor");
    if (!raw.empty()) std::memcpy(dst, raw.data(), raw.size());
    return ZJAI_OK;
  } catch (const std::bad_alloc&) {
    return fail(ZJAI_LIMIT_EXCEEDED, "checkpoint: out of host memory");
  }
}

int zjai_ckpt_int(const zjai_ckpt* ck, int i, const char** name, int64_t* value) {
  if (!ck || i < 0 || i >= (int)ck->ints.size())
    return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: integer index out of range");
  if (name) *name = ck->ints[i].first.c_str();
  if (value) *value = ck->ints[i].second;
  return ZJAI_OK;
}

int zjai_ckpt_list(const zjai_ckpt* ck, int i, const char** name, const double** values, int* n) {
  if (!ck || i < 0 || i >= (int)ck->lists.size())
    return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: list index out of range");
  if (name) *name = ck->lists[i].first.c_str();
  if (values) *values = ck->lists[i].second.data();
  if (n) *n = (int)ck->lists[i].second.size();
  return ZJAI_OK;
}

int zjai_ckpt_params(zjai_ckpt* ck, const zjai_param** params, int* n) {
  if (!ck || !params || !n) return fail(ZJAI_INVALID_ARGUMENT, "checkpoint: bad arguments");
  try {
    ZJAI_TRY(wio::build_params(ck));
  } catch (const std::bad_alloc&) {
    return fail(ZJAI_LIMIT_EXCEEDED, "checkpoint: out of host memory");
  }
  *params = ck->params.data();
  *n = (int)ck->params.size();
  return ZJAI_OK;
}

int zjai_bundle_open(const void* data, size_t len, zjai_bundle** out) {
  if (!out) return fail(ZJAI_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  const uint8_t* p = static_cast<const uint8_t*>(data);
  if (!p || len < 4 || (std::memcmp(p, "ZJB1", 4) != 0 && std::memcmp(p, "ZJB2", 4) != 0))
    return fail(ZJAI_MODEL, "bundle: bad magic");
  try {
    std::unique_ptr<zjai_bundle> b(new zjai_bundle());
    b->file.assign(p, p + len);
    b->f16 = p[3] == '2';
    ZJAI_TRY(wio::parse_bundle(b.get()));
    *out = b.release();
    return ZJAI_OK;
  } catch (const std::bad_alloc&) {
    return fail(ZJAI_LIMIT_EXCEEDED, "bundle: out of host memory");
  }
}

int zjai_bundle_close(zjai_bundle* b) {
  delete b;
  return ZJAI_OK;
}

int zjai_bundle_info(const zjai_bundle* b, int* nfiles, int* f16, const char** notice,
                     size_t* notice_len) {
  if (!b) return fail(ZJAI_INVALID_ARGUMENT, "null bundle");
  if (nfiles) *nfiles = (int)b->files.size();
  if (f16) *f16 = b->f16 ? 1 : 0;
  if (notice) *notice = b->notice.data();
  if (notice_len) *notice_len = b->notice.size();
  return ZJAI_OK;
}

int zjai_bundle_file(const zjai_bundle* b, int i, const char** path, const void** data,
                     size_t* len) {
  if (!b || i < 0 || i >= (int)b->files.size())
    return fail(ZJAI_INVALID_ARGUMENT, "bundle: file index out of range");
  if (path) *path = b->files[i].first.c_str();
  if (data) *data = b->file.data() + b->files[i].second.off;
  if (len) *len = b->files[i].second.len;
  return ZJAI_OK;
}
