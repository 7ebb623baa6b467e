// Minimal stand-in for the glog assertions the KVM front end uses (CHECK,
// CHECK_EQ): glog is not installed on these machines. A failed check prints
// the file, line, condition and streamed message to stderr and aborts, as
// glog's CHECK does.
#pragma once

#include <cstdlib>
#include <iostream>
#include <sstream>

namespace kvm_glog_shim {

class FatalMessage {
 public:
  FatalMessage(const char* file, int line, const char* cond) {
    os_ << file << ":" << line << "] Check failed: " << cond << " ";
  }
  [[noreturn]] ~FatalMessage() {
    std::cerr << os_.str() << std::endl;
    std::abort();
  }
  std::ostream& stream() { return os_; }

 private:
  std::ostringstream os_;
};

// Swallows the stream when the check passes.
struct Voidify {
  void operator&(std::ostream&) {}
};

}  // namespace kvm_glog_shim

#define CHECK(cond)                                                    \
  (cond) ? (void)0                                                     \
         : ::kvm_glog_shim::Voidify() &                                \
               ::kvm_glog_shim::FatalMessage(__FILE__, __LINE__, #cond) \
                   .stream()

#define CHECK_EQ(a, b) CHECK((a) == (b))
#define CHECK_NE(a, b) CHECK((a) != (b))

namespace google {
inline void InitGoogleLogging(const char*) {}
inline void LogToStderr() {}
}  // namespace google
