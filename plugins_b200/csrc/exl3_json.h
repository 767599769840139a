// exl3_json.h -- a small JSON reader for config blocks and config.json (host code): values, no streaming.
#pragma once
#include <cstdio>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "../../include/exl3_b200.h"

namespace exl3 {

struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  bool is_int = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* key) const {
    if (kind != Obj) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* end;
  int depth = 0;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if (static_cast<size_t>(end - p) < n || strncmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  bool string(std::string& out) {
    if (p >= end || *p != '"') return false;
    ++p;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= end) return false;
        char c = *p++;
        switch (c) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (end - p < 4) return false;
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= h - '0';
              else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
              else return false;
            }
            out += static_cast<char>(v < 0x80 ? v : '?');
            break;
          }
          default: out += c;
        }
      } else {
        out += *p++;
      }
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool value(JVal& v) {
    if (++depth > 64) return false;
    ws();
    if (p >= end) return false;
    bool ok = true;
    if (*p == '{') {
      v.kind = JVal::Obj;
      ++p;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        while (true) {
          ws();
          std::string key;
          if (!string(key)) { ok = false; break; }
          ws();
          if (p >= end || *p != ':') { ok = false; break; }
          ++p;
          JVal child;
          if (!value(child)) { ok = false; break; }
          v.obj.emplace_back(std::move(key), std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == '}') { ++p; break; }
          ok = false;
          break;
        }
      }
    } else if (*p == '[') {
      v.kind = JVal::Arr;
      ++p;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        while (true) {
          JVal child;
          if (!value(child)) { ok = false; break; }
          v.arr.push_back(std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == ']') { ++p; break; }
          ok = false;
          break;
        }
      }
    } else if (*p == '"') {
      v.kind = JVal::Str;
      ok = string(v.str);
    } else if (lit("true")) {
      v.kind = JVal::Bool;
      v.b = true;
    } else if (lit("false")) {
      v.kind = JVal::Bool;
    } else if (lit("null")) {
      v.kind = JVal::Null;
    } else {
      const char* s = p;
      while (p < end && (isdigit(static_cast<unsigned char>(*p)) || *p == '-' || *p == '+' || *p == '.' || *p == 'e' || *p == 'E')) ++p;
      if (p == s) return false;
      std::string t(s, p);
      char* e = nullptr;
      v.kind = JVal::Num;
      v.num = strtod(t.c_str(), &e);
      v.is_int = t.find_first_of(".eE") == std::string::npos;
      ok = e && *e == 0;
    }
    --depth;
    return ok;
  }
};

inline bool parse_json(exl3_str s, JVal& out) {
  if (!s.ptr) return false;
  JParser jp{s.ptr, s.ptr + s.len};
  if (!jp.value(out)) return false;
  jp.ws();
  return jp.p == jp.end;
}

inline bool str_is(const JVal* v, const char* s) { return v && v->kind == JVal::Str && v->str == s; }

// The value as JSON text (the blocks a load hands to exl3_open); numbers keep their integer form where they had one.
inline void dump_json(const JVal& v, std::string& out) {
  switch (v.kind) {
    case JVal::Null: out += "null"; break;
    case JVal::Bool: out += v.b ? "true" : "false"; break;
    case JVal::Num: {
      char buf[40];
      if (v.is_int) snprintf(buf, sizeof buf, "%lld", static_cast<long long>(v.num));
      else snprintf(buf, sizeof buf, "%.17g", v.num);
      out += buf;
      break;
    }
    case JVal::Str:
      out += '"';
      for (char c : v.str) {
        if (static_cast<unsigned char>(c) < 0x20) {
          char esc[8];
          snprintf(esc, sizeof esc, "\\u%04x", static_cast<unsigned>(static_cast<unsigned char>(c)));
          out += esc;
          continue;
        }
        if (c == '"' || c == '\\') out += '\\';
        out += c;
      }
      out += '"';
      break;
    case JVal::Arr:
      out += '[';
      for (size_t i = 0; i < v.arr.size(); ++i) {
        if (i) out += ',';
        dump_json(v.arr[i], out);
      }
      out += ']';
      break;
    case JVal::Obj:
      out += '{';
      for (size_t i = 0; i < v.obj.size(); ++i) {
        if (i) out += ',';
        JVal k;
        k.kind = JVal::Str;
        k.str = v.obj[i].first;
        dump_json(k, out);
        out += ':';
        dump_json(v.obj[i].second, out);
      }
      out += '}';
      break;
  }
}

}  // namespace exl3
