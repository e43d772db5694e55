// expr.cpp — host compiler of registered expression operators.
//
// The reference compiles each `register_elementwise(key, expr, arity)` expression with
// NVRTC into its own module (pytorch_ext/gpuos_ext.cpp:814-881).  Here the expression is
// parsed once on the host into a postfix program for the worker's stack machine
// (device/expr.cuh): C float expressions over A and B — literals (`0.5`, `1.f`, `1e-3f`),
// `+ - * /`, comparisons, `! && ||`, `?:`, parentheses, `(float)` casts and the float
// functions listed in kUnary/kBinary (with or without the `f` suffix).  Operator precedence
// and associativity follow C.
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "internal.h"

namespace gpuos {
namespace {

struct Fn {
  const char* name;
  uint8_t op;
};
const Fn kUnary[] = {{"exp", XO_EXP},     {"log", XO_LOG},     {"log1p", XO_LOG1P}, {"expm1", XO_EXPM1},
                     {"sqrt", XO_SQRT},   {"rsqrt", XO_RSQRT}, {"fabs", XO_ABS},    {"abs", XO_ABS},
                     {"tanh", XO_TANH},   {"sin", XO_SIN},     {"cos", XO_COS},     {"tan", XO_TAN},
                     {"erf", XO_ERF},     {"floor", XO_FLOOR}, {"ceil", XO_CEIL},   {"trunc", XO_TRUNC},
                     {"round", XO_ROUND}, {"exp2", XO_EXP2},   {"log2", XO_LOG2},   {"log10", XO_LOG10},
                     {"sinh", XO_SINH},   {"cosh", XO_COSH},   {"asin", XO_ASIN},   {"acos", XO_ACOS},
                     {"atan", XO_ATAN}};
const Fn kBinary[] = {{"fmin", XO_MIN}, {"min", XO_MIN},   {"fmax", XO_MAX},     {"max", XO_MAX},
                      {"pow", XO_POW},  {"fmod", XO_FMOD}, {"atan2", XO_ATAN2}, {"copysign", XO_COPYSIGN}};

class Parser {
 public:
  Parser(const char* src, int arity, ExprProg* out) : s_(src), arity_(arity), p_(out) {}

  bool run(std::string* err) {
    std::memset(p_, 0, sizeof(*p_));
    if (!ternary()) {
      *err = err_;
      return false;
    }
    skip();
    if (s_[pos_] != '\0') {
      *err = at("unexpected '" + std::string(1, s_[pos_]) + "'");
      return false;
    }
    if (depth_ != 1) {
      *err = "internal: unbalanced program";
      return false;
    }
    p_->len = len_;
    p_->arity = arity_;
    p_->depth = max_depth_;
    return true;
  }

 private:
  const char* s_;
  int arity_;
  ExprProg* p_;
  size_t pos_ = 0;
  int len_ = 0, depth_ = 0, max_depth_ = 0;
  std::string err_;

  std::string at(const std::string& what) const { return what + " at column " + std::to_string(pos_ + 1); }
  bool fail(const std::string& what) {
    if (err_.empty()) err_ = at(what);
    return false;
  }
  void skip() {
    while (std::isspace((unsigned char)s_[pos_])) ++pos_;
  }
  bool peek(const char* tok) {
    skip();
    return std::strncmp(s_ + pos_, tok, std::strlen(tok)) == 0;
  }
  bool accept(const char* tok) {
    if (!peek(tok)) return false;
    pos_ += std::strlen(tok);
    return true;
  }
  // emit: `pops` operands consumed, one result pushed
  bool emit(uint8_t op, int pops, float imm = 0.f) {
    if (len_ >= kExprMaxCode) return fail("expression longer than " + std::to_string(kExprMaxCode) + " steps");
    p_->code[len_] = op;
    p_->imm[len_] = imm;
    ++len_;
    depth_ += 1 - pops;
    if (depth_ > max_depth_) max_depth_ = depth_;
    if (max_depth_ > kExprMaxStack) return fail("expression nests deeper than " + std::to_string(kExprMaxStack));
    return true;
  }

  bool ternary() {
    if (!logic_or()) return false;
    if (!accept("?")) return true;
    if (!ternary()) return false;
    if (!accept(":")) return fail("expected ':'");
    if (!ternary()) return false;
    return emit(XO_SELECT, 3);
  }
  bool logic_or() {
    if (!logic_and()) return false;
    while (accept("||")) {
      if (!logic_and() || !emit(XO_OR, 2)) return false;
    }
    return true;
  }
  bool logic_and() {
    if (!equality()) return false;
    while (accept("&&")) {
      if (!equality() || !emit(XO_AND, 2)) return false;
    }
    return true;
  }
  bool equality() {
    if (!relational()) return false;
    while (true) {
      uint8_t op;
      if (accept("==")) op = XO_EQ;
      else if (accept("!=")) op = XO_NE;
      else return true;
      if (!relational() || !emit(op, 2)) return false;
    }
  }
  bool relational() {
    if (!additive()) return false;
    while (true) {
      uint8_t op;
      if (accept("<=")) op = XO_LE;
      else if (accept(">=")) op = XO_GE;
      else if (accept("<")) op = XO_LT;
      else if (accept(">")) op = XO_GT;
      else return true;
      if (!additive() || !emit(op, 2)) return false;
    }
  }
  bool additive() {
    if (!multiplicative()) return false;
    while (true) {
      uint8_t op;
      if (accept("+")) op = XO_ADD;
      else if (accept("-")) op = XO_SUB;
      else return true;
      if (!multiplicative() || !emit(op, 2)) return false;
    }
  }
  bool multiplicative() {
    if (!unary()) return false;
    while (true) {
      uint8_t op;
      if (accept("*")) op = XO_MUL;
      else if (accept("/")) op = XO_DIV;
      else return true;
      if (!unary() || !emit(op, 2)) return false;
    }
  }
  bool unary() {
    if (accept("-")) return unary() && emit(XO_NEG, 1);
    if (accept("+")) return unary();
    if (peek("!") && !peek("!=")) {
      accept("!");
      return unary() && emit(XO_NOT, 1);
    }
    // C cast to float: a no-op on float values
    skip();
    const size_t save = pos_;
    if (accept("(")) {
      skip();
      if (std::strncmp(s_ + pos_, "float", 5) == 0) {
        pos_ += 5;
        if (accept(")")) return unary();
      }
      pos_ = save;
    }
    return primary();
  }
  bool primary() {
    skip();
    const char c = s_[pos_];
    if (c == '(') {
      ++pos_;
      if (!ternary()) return false;
      if (!accept(")")) return fail("expected ')'");
      return true;
    }
    if (std::isdigit((unsigned char)c) || (c == '.' && std::isdigit((unsigned char)s_[pos_ + 1]))) return number();
    if (std::isalpha((unsigned char)c) || c == '_') {
      size_t e = pos_;
      while (std::isalnum((unsigned char)s_[e]) || s_[e] == '_') ++e;
      std::string id(s_ + pos_, e - pos_);
      pos_ = e;
      if (id == "A") return emit(XO_A, 0);
      if (id == "B") {
        if (arity_ != 2) return fail("B used in a one-operand expression");
        return emit(XO_B, 0);
      }
      return call(id);
    }
    if (c == '\0') return fail("expression ends early");
    return fail("unexpected '" + std::string(1, c) + "'");
  }
  bool number() {
    const char* begin = s_ + pos_;
    char* end = nullptr;
    const double v = std::strtod(begin, &end);
    if (end == begin) return fail("bad number");
    pos_ += (size_t)(end - begin);
    if (s_[pos_] == 'f' || s_[pos_] == 'F') ++pos_;
    return emit(XO_CONST, 0, (float)v);
  }
  bool call(const std::string& raw) {
    std::string name = raw;
    // the C float spellings (expf, fmaxf, ...) name the same functions
    const Fn* hit = nullptr;
    int nargs = 0;
    for (int pass = 0; pass < 2 && !hit; ++pass) {
      for (const Fn& f : kUnary)
        if (name == f.name) hit = &f, nargs = 1;
      for (const Fn& f : kBinary)
        if (name == f.name) hit = &f, nargs = 2;
      if (!hit && name.size() > 1 && name.back() == 'f') name.pop_back();
      else break;
    }
    if (!hit) return fail("unknown function '" + raw + "'");
    if (!accept("(")) return fail("expected '(' after " + raw);
    if (!ternary()) return false;
    if (nargs == 2) {
      if (!accept(",")) return fail(raw + " takes two arguments");
      if (!ternary()) return false;
    }
    if (!accept(")")) return fail("expected ')' after the arguments of " + raw);
    return emit(hit->op, nargs);
  }
};

}  // namespace

int expr_compile(const char* expr, int arity, ExprProg* out, std::string* err) {
  if (!expr || !out) {
    *err = "null argument";
    return GPUOS_ERR_INVALID;
  }
  if (arity != 1 && arity != 2) {
    *err = "arity must be 1 or 2";
    return GPUOS_ERR_INVALID;
  }
  Parser p(expr, arity, out);
  if (!p.run(err)) return GPUOS_ERR_INVALID;
  return GPUOS_OK;
}

}  // namespace gpuos
