// PGW1 parser: header layout engine/weights.js:5-40, writer tools/convert_hf_to_pgw.py:123-144.
// The tensor table is JSON; this reader accepts the subset the converters emit (an array of flat
// objects whose values are strings, numbers or arrays of numbers) and rejects anything else.
#include "pgw.hpp"

#include <cstring>

namespace mllm {
namespace {

struct Json {
  const char* p;
  const char* end;
  std::string err;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool expect(char c) {
    ws();
    if (p < end && *p == c) {
      ++p;
      return true;
    }
    err = std::string("expected '") + c + "'";
    return false;
  }
  bool peek(char c) {
    ws();
    return p < end && *p == c;
  }
  bool str(std::string* out) {
    if (!expect('"')) return false;
    out->clear();
    while (p < end && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= end) break;
        switch (*p) {
          case 'n': out->push_back('\n'); break;
          case 't': out->push_back('\t'); break;
          case 'u': {  // keep ASCII escapes, replace others; names are ASCII in practice
            if (end - p < 5) { err = "bad escape"; return false; }
            unsigned v = 0;
            for (int i = 1; i <= 4; ++i) {
              char h = p[i];
              v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : (h | 32) - 'a' + 10);
            }
            out->push_back(v < 128 ? (char)v : '?');
            p += 4;
            break;
          }
          default: out->push_back(*p);
        }
        ++p;
      } else {
        out->push_back(*p++);
      }
    }
    if (p >= end) { err = "unterminated string"; return false; }
    ++p;
    return true;
  }
  bool num(double* out) {
    ws();
    const char* s = p;
    while (p < end && (strchr("+-0123456789.eE", *p) != nullptr)) ++p;
    if (p == s) { err = "expected number"; return false; }
    *out = strtod(std::string(s, p).c_str(), nullptr);
    return true;
  }
  bool skip_literal() {  // true / false / null
    ws();
    for (const char* lit : {"true", "false", "null"}) {
      size_t n = strlen(lit);
      if ((size_t)(end - p) >= n && strncmp(p, lit, n) == 0) {
        p += n;
        return true;
      }
    }
    err = "unexpected value";
    return false;
  }
};

uint32_t rd32(const uint8_t* b) { uint32_t v; memcpy(&v, b, 4); return v; }
double rdf64(const uint8_t* b) { double v; memcpy(&v, b, 8); return v; }

}  // namespace

bool parse_pgw(const uint8_t* buf, size_t len, PgwModel* m, std::string* err) {
  if (!buf || len < 256) { *err = "truncated PGW1 header"; return false; }
  if (memcmp(buf, "PGW1", 4) != 0) {
    *err = std::string("bad magic ") + std::string((const char*)buf, 4);
    return false;
  }
  static const char* kinds[] = {"f32", "f16", "bf16", "q8", "q4"};  // engine/weights.js:3
  m->kind = buf[4] < 5 ? kinds[buf[4]] : "f32";
  m->arch = buf[5] == 1 ? 1 : 0;
  m->vocab = (int)rd32(buf + 8);
  m->n_layers = (int)rd32(buf + 12);
  m->d_model = (int)rd32(buf + 16);
  m->n_heads = (int)rd32(buf + 20);
  m->n_kv_heads = (int)rd32(buf + 24);
  m->d_ff = (int)rd32(buf + 28);
  m->max_seq = (int)rd32(buf + 32);
  m->q_group = rd32(buf + 36) ? (int)rd32(buf + 36) : 32;
  m->rope_theta = rdf64(buf + 56) != 0.0 ? rdf64(buf + 56) : 10000.0;
  m->rope_pct = rdf64(buf + 64) != 0.0 ? rdf64(buf + 64) : 1.0;
  const uint32_t toff = rd32(buf + 40), tlen = rd32(buf + 44);
  m->payload_off = rd32(buf + 48);
  if ((uint64_t)toff + tlen > len) { *err = "truncated PGW1 tensor table"; return false; }
  Json j{(const char*)buf + toff, (const char*)buf + toff + tlen, ""};
  if (!j.expect('[')) { *err = "tensor table: " + j.err; return false; }
  bool first = true;
  while (!j.peek(']')) {
    if (!first && !j.expect(',')) { *err = "tensor table: " + j.err; return false; }
    first = false;
    if (!j.expect('{')) { *err = "tensor table: " + j.err; return false; }
    PgwTensor t;
    bool kfirst = true;
    while (!j.peek('}')) {
      if (!kfirst && !j.expect(',')) { *err = "tensor table: " + j.err; return false; }
      kfirst = false;
      std::string key;
      if (!j.str(&key) || !j.expect(':')) { *err = "tensor table: " + j.err; return false; }
      j.ws();
      if (j.peek('"')) {
        std::string v;
        if (!j.str(&v)) { *err = "tensor table: " + j.err; return false; }
        if (key == "name") t.name = v;
        else if (key == "storage") t.storage = v;
      } else if (j.peek('[')) {
        j.expect('[');
        std::vector<int64_t> dims;
        while (!j.peek(']')) {
          if (!dims.empty() && !j.expect(',')) { *err = "tensor table: " + j.err; return false; }
          double d;
          if (!j.num(&d)) { *err = "tensor table: " + j.err; return false; }
          dims.push_back((int64_t)d);
        }
        j.expect(']');
        if (key == "shape") t.shape = dims;
      } else if (j.peek('t') || j.peek('f') || j.peek('n')) {
        if (!j.skip_literal()) { *err = "tensor table: " + j.err; return false; }
      } else {
        double d;
        if (!j.num(&d)) { *err = "tensor table: " + j.err; return false; }
        const int64_t v = (int64_t)d;
        if (key == "group") t.group = (int)v;
        else if (key == "offset") t.offset = v;
        else if (key == "nbytes") t.nbytes = v;
        else if (key == "scaleOffset") t.scale_offset = v;
        else if (key == "scaleNbytes") t.scale_nbytes = v;
      }
    }
    j.expect('}');
    if (t.name.empty()) { *err = "tensor table: entry without a name"; return false; }
    if (t.group == 0) t.group = 32;
    const uint64_t end = (uint64_t)m->payload_off + t.offset + t.nbytes;
    if (t.offset < 0 || t.nbytes < 0 || end > len) { *err = "tensor " + t.name + " lies outside the file"; return false; }
    if (t.storage == "q4") {
      const uint64_t send = (uint64_t)m->payload_off + t.scale_offset + t.scale_nbytes;
      if (t.scale_offset < 0 || send > len) { *err = "scales of " + t.name + " lie outside the file"; return false; }
    }
    m->tensors[t.name] = t;
  }
  // engine/weights.js:36-38
  if (m->arch == 1 && !m->tensors.count("blocks.0.ln1") && m->tensors.count("blocks.0.norm1")) m->arch = 0;
  return true;
}

}  // namespace mllm
