// Debug aid: a SIGSEGV/SIGBUS handler that prints the native backtrace of the
// faulting thread to stderr (installed on request only).
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>

namespace mtorus {

static void segv_handler(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char msg[] = "\n[mtorus] fatal signal, native backtrace:\n";
  ssize_t w = write(2, msg, sizeof(msg) - 1);
  (void)w;
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}

void install_segv_handler() {
  signal(SIGSEGV, segv_handler);
  signal(SIGBUS, segv_handler);
}

}  // namespace mtorus
