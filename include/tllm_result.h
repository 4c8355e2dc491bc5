// tiny_llm::Result<T> for builds of this library's C++ facade that do not
// have tiny-llm's own headers (the facade's tests, standalone users).
//
// Inside the tiny-llm engine tree, include/tiny_llm/kv_cache.h uses the
// engine's own tiny_llm/result.h instead and this file is never included, so
// the two definitions never meet. The interface is kept alike with the
// reference's include/tiny_llm/result.h:11-112 (ok/err factories,
// isOk/isErr, value() that throws on error, error() that throws on ok,
// valueOr, map, flatMap with ValueType, and a Result<void> specialisation) so
// code written against tiny-llm's KVCacheManager compiles with either.
#pragma once

#include <stdexcept>
#include <string>
#include <utility>
#include <variant>

namespace tiny_llm {

template <typename T>
class Result {
  public:
    using ValueType = T;

    static Result ok(T value) { return Result(std::in_place_index<0>, std::move(value)); }
    static Result err(std::string message) { return Result(std::in_place_index<1>, std::move(message)); }

    bool isOk() const { return state_.index() == 0; }
    bool isErr() const { return !isOk(); }

    T &value() {
        if (isErr()) throw std::runtime_error("Attempted to access value of error Result: " + error());
        return std::get<0>(state_);
    }
    const T &value() const {
        if (isErr()) throw std::runtime_error("Attempted to access value of error Result: " + error());
        return std::get<0>(state_);
    }
    const std::string &error() const {
        if (isOk()) throw std::runtime_error("Attempted to access error of ok Result");
        return std::get<1>(state_);
    }
    T valueOr(T fallback) const { return isOk() ? std::get<0>(state_) : std::move(fallback); }

    // f(T) -> U; an error passes through with its message.
    template <typename F>
    auto map(F &&f) -> Result<decltype(f(std::declval<T>()))> {
        using U = decltype(f(std::declval<T>()));
        if (isErr()) return Result<U>::err(error());
        return Result<U>::ok(f(value()));
    }

    // f(T) -> Result<U>; an error passes through with its message.
    template <typename F>
    auto flatMap(F &&f) -> decltype(f(std::declval<T>())) {
        using R = decltype(f(std::declval<T>()));
        if (isErr()) return R::err(error());
        return f(value());
    }

  private:
    template <std::size_t I, typename U>
    Result(std::in_place_index_t<I> tag, U &&u) : state_(tag, std::forward<U>(u)) {}
    std::variant<T, std::string> state_;
};

template <>
class Result<void> {
  public:
    static Result ok() { return Result(true, std::string()); }
    static Result err(std::string message) { return Result(false, std::move(message)); }

    bool isOk() const { return ok_; }
    bool isErr() const { return !ok_; }
    const std::string &error() const {
        if (ok_) throw std::runtime_error("Attempted to access error of ok Result");
        return message_;
    }

  private:
    Result(bool ok, std::string m) : ok_(ok), message_(std::move(m)) {}
    bool ok_;
    std::string message_;
};

}  // namespace tiny_llm
