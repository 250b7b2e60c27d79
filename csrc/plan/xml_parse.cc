// Minimal XML reader for MSCCL algorithm files.
//
// The files contain only elements with attributes (<algo>, <gpu>, <tb>,
// <step>), optional declarations and comments.  The reader builds the element
// tree, then maps it onto XAlgo with strict integer attribute checks.
#include <cctype>
#include <cstring>
#include <cstdlib>
#include <memory>
#include <string>
#include <vector>

#include "vb/plan.h"

namespace vb {
namespace {

struct Element {
  std::string name;
  std::vector<std::pair<std::string, std::string>> attrs;
  std::vector<std::unique_ptr<Element>> children;

  const std::string* attr(const char* key) const {
    for (auto& kv : attrs)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class Reader {
 public:
  explicit Reader(const std::string& t) : s_(t) {}

  std::unique_ptr<Element> parse() {
    std::unique_ptr<Element> root;
    std::vector<Element*> stack;
    while (true) {
      skip_text();
      if (pos_ >= s_.size()) break;
      if (starts("<?")) { skip_until("?>"); continue; }
      if (starts("<!--")) { skip_until("-->"); continue; }
      if (starts("<!")) { skip_until(">"); continue; }
      if (starts("</")) {
        pos_ += 2;
        std::string name = ident();
        skip_ws();
        expect('>');
        if (stack.empty() || stack.back()->name != name) fail("mismatched closing tag </" + name + ">");
        stack.pop_back();
        continue;
      }
      expect('<');
      auto el = std::make_unique<Element>();
      el->name = ident();
      bool self_closing = false;
      while (true) {
        skip_ws();
        if (starts("/>")) { pos_ += 2; self_closing = true; break; }
        if (starts(">")) { pos_ += 1; break; }
        std::string key = ident();
        skip_ws();
        expect('=');
        skip_ws();
        char q = peek();
        if (q != '"' && q != '\'') fail("attribute value must be quoted");
        ++pos_;
        size_t end = s_.find(q, pos_);
        if (end == std::string::npos) fail("unterminated attribute value");
        std::string value = unescape(s_.substr(pos_, end - pos_));
        pos_ = end + 1;
        for (auto& kv : el->attrs)
          if (kv.first == key) fail("duplicate attribute " + key);
        el->attrs.emplace_back(key, value);
      }
      Element* raw = el.get();
      if (stack.empty()) {
        if (root) fail("more than one root element");
        root = std::move(el);
      } else {
        stack.back()->children.push_back(std::move(el));
      }
      if (!self_closing) stack.push_back(raw);
    }
    if (!stack.empty()) fail("unclosed element <" + stack.back()->name + ">");
    if (!root) fail("empty document");
    return root;
  }

 private:
  [[noreturn]] void fail(const std::string& m) { throw CompileError("xml: " + m + " at offset " + std::to_string(pos_)); }
  bool starts(const char* p) const { return s_.compare(pos_, strlen(p), p) == 0; }
  char peek() const { return pos_ < s_.size() ? s_[pos_] : '\0'; }
  void expect(char c) {
    if (peek() != c) fail(std::string("expected '") + c + "'");
    ++pos_;
  }
  void skip_ws() { while (pos_ < s_.size() && std::isspace((unsigned char)s_[pos_])) ++pos_; }
  void skip_text() { while (pos_ < s_.size() && s_[pos_] != '<') ++pos_; }
  void skip_until(const char* end) {
    size_t e = s_.find(end, pos_);
    if (e == std::string::npos) fail(std::string("unterminated construct, missing ") + end);
    pos_ = e + strlen(end);
  }
  std::string ident() {
    size_t b = pos_;
    while (pos_ < s_.size() && (std::isalnum((unsigned char)s_[pos_]) || s_[pos_] == '_' || s_[pos_] == '-' ||
                                s_[pos_] == ':' || s_[pos_] == '.'))
      ++pos_;
    if (b == pos_) fail("expected a name");
    return s_.substr(b, pos_ - b);
  }
  static std::string unescape(const std::string& v) {
    std::string out;
    for (size_t i = 0; i < v.size(); ++i) {
      if (v[i] == '&') {
        size_t e = v.find(';', i);
        std::string ent = e == std::string::npos ? "" : v.substr(i + 1, e - i - 1);
        if (ent == "lt") out += '<'; else if (ent == "gt") out += '>'; else if (ent == "amp") out += '&';
        else if (ent == "quot") out += '"'; else if (ent == "apos") out += '\'';
        else { out += v[i]; continue; }
        i = e;
      } else {
        out += v[i];
      }
    }
    return out;
  }
  const std::string& s_;
  size_t pos_ = 0;
};

long long to_int(const Element& el, const char* key, bool required, long long dflt) {
  const std::string* v = el.attr(key);
  if (!v) {
    if (required) throw CompileError("xml: <" + el.name + "> lacks attribute " + key);
    return dflt;
  }
  char* end = nullptr;
  long long x = std::strtoll(v->c_str(), &end, 10);
  if (v->empty() || *end != '\0') throw CompileError("xml: attribute " + std::string(key) + "='" + *v + "' is not an integer");
  return x;
}

int buf_code(const Element& el, const char* key) {
  const std::string* v = el.attr(key);
  if (!v) return BUF_IN;
  if (*v == "i") return BUF_IN;
  if (*v == "o") return BUF_OUT;
  if (*v == "s") return BUF_SCR;
  throw CompileError("xml: unknown buffer '" + *v + "'");
}

XKind kind_code(const std::string& t) {
  if (t == "s") return X_S;
  if (t == "r") return X_R;
  if (t == "rrc") return X_RRC;
  if (t == "rcs") return X_RCS;
  if (t == "rrs") return X_RRS;
  if (t == "rrcs") return X_RRCS;
  if (t == "cpy") return X_CPY;
  if (t == "re") return X_RE;
  if (t == "nop") return X_NOP;
  throw CompileError("xml: unknown step type '" + t + "'");
}

}  // namespace

XAlgo parse_xml(const std::string& text) {
  Reader reader(text);
  auto root = reader.parse();
  if (root->name != "algo") throw CompileError("xml: root element must be <algo>");
  XAlgo a;
  auto str = [&](const char* k, const char* d) { const std::string* v = root->attr(k); return v ? *v : std::string(d); };
  a.name = str("name", "algo");
  a.proto = str("proto", "Simple");
  a.coll = str("coll", "allreduce");
  a.redop = str("redop", "nop");
  a.nchannels = (int)to_int(*root, "nchannels", false, 1);
  a.nchunksperloop = (int)to_int(*root, "nchunksperloop", true, 0);
  a.inplace = (int)to_int(*root, "inplace", false, 0);
  a.ngpus = (int)to_int(*root, "ngpus", true, 0);
  a.min_bytes = to_int(*root, "minBytes", false, 0);
  a.max_bytes = to_int(*root, "maxBytes", false, 0);
  if (a.ngpus < 1 || a.ngpus > kMaxRanks) throw CompileError("xml: ngpus must be in [1, 16]");
  if (a.nchunksperloop < 1) throw CompileError("xml: nchunksperloop must be positive");
  a.gpus.resize(a.ngpus);
  std::vector<bool> seen(a.ngpus, false);
  for (auto& g : root->children) {
    if (g->name != "gpu") throw CompileError("xml: <algo> may only contain <gpu>");
    int id = (int)to_int(*g, "id", true, 0);
    if (id < 0 || id >= a.ngpus || seen[id]) throw CompileError("xml: invalid or duplicate gpu id");
    seen[id] = true;
    XGpu& gpu = a.gpus[id];
    gpu.id = id;
    gpu.i_chunks = (int)to_int(*g, "i_chunks", false, 0);
    gpu.o_chunks = (int)to_int(*g, "o_chunks", false, 0);
    gpu.s_chunks = (int)to_int(*g, "s_chunks", false, 0);
    for (auto& t : g->children) {
      if (t->name != "tb") throw CompileError("xml: <gpu> may only contain <tb>");
      XTB tb;
      tb.id = (int)to_int(*t, "id", true, 0);
      tb.send = (int)to_int(*t, "send", false, -1);
      tb.recv = (int)to_int(*t, "recv", false, -1);
      tb.chan = (int)to_int(*t, "chan", false, 0);
      int index = 0;
      for (auto& s : t->children) {
        if (s->name != "step") throw CompileError("xml: <tb> may only contain <step>");
        if (to_int(*s, "s", true, 0) != index) throw CompileError("xml: step indices must be dense and ordered");
        const std::string* ty = s->attr("type");
        if (!ty) throw CompileError("xml: step lacks type");
        XStep st;
        st.kind = kind_code(*ty);
        st.srcbuf = buf_code(*s, "srcbuf");
        st.srcoff = (int)to_int(*s, "srcoff", false, -1);
        st.dstbuf = buf_code(*s, "dstbuf");
        st.dstoff = (int)to_int(*s, "dstoff", false, -1);
        st.cnt = (int)to_int(*s, "cnt", false, 1);
        st.depid = (int)to_int(*s, "depid", false, -1);
        st.deps = (int)to_int(*s, "deps", false, -1);
        st.hasdep = (int)to_int(*s, "hasdep", false, 0);
        if (st.cnt < 1) throw CompileError("xml: cnt must be positive");
        tb.steps.push_back(st);
        ++index;
      }
      gpu.tbs.push_back(std::move(tb));
    }
  }
  for (int r = 0; r < a.ngpus; ++r)
    if (!seen[r]) a.gpus[r].id = r;
  return a;
}

}  // namespace vb
