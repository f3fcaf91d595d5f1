// marketforge::Result<T> — value-or-Status, the reference's shape
// (include/marketforge/core/result.hpp:12-57).
#pragma once

#include <cassert>
#include <type_traits>
#include <utility>
#include <variant>

#include "marketforge/core/status.hpp"

namespace marketforge {

template <typename T>
class [[nodiscard]] Result {
  static_assert(!std::is_same_v<std::remove_cv_t<T>, Status>);

 public:
  [[nodiscard]] static Result success(T value) { return Result(std::in_place_index<0>, std::move(value)); }
  [[nodiscard]] static Result failure(Status status) {
    assert(!status.ok());
    return Result(std::in_place_index<1>, status);
  }
  [[nodiscard]] bool has_value() const noexcept { return storage_.index() == 0; }
  [[nodiscard]] explicit operator bool() const noexcept { return has_value(); }
  [[nodiscard]] T& value() & { return std::get<0>(storage_); }
  [[nodiscard]] const T& value() const& { return std::get<0>(storage_); }
  [[nodiscard]] T&& value() && { return std::get<0>(std::move(storage_)); }
  [[nodiscard]] Status status() const noexcept {
    return has_value() ? Status::success() : std::get<1>(storage_);
  }

 private:
  template <std::size_t I, typename V>
  explicit Result(std::in_place_index_t<I> i, V&& v) : storage_(i, std::forward<V>(v)) {}
  std::variant<T, Status> storage_;
};

}  // namespace marketforge
