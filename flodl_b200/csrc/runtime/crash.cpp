// Native crash reporter: on SIGSEGV/SIGBUS/SIGILL/SIGFPE print the faulting
// address and the native call stack (module + offset, resolvable with
// addr2line against the in-tree .so files), then hand the signal to the
// handler that was installed before (e.g. Python's faulthandler, which adds
// the Python stacks) so the process still dies with the original signal.
#include <dlfcn.h>
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>

#include "runtime.h"

namespace flodl {
namespace rt {
namespace {

constexpr int kSignals[] = {SIGSEGV, SIGBUS, SIGILL, SIGFPE};
struct sigaction g_prev[4];
volatile sig_atomic_t g_installed = 0;

int slot_of(int sig) {
  for (int i = 0; i < 4; ++i)
    if (kSignals[i] == sig) return i;
  return -1;
}

void on_fatal(int sig, siginfo_t* si, void* /*ctx*/) {
  char buf[160];
  int n = snprintf(buf, sizeof(buf), "\nflodl_b200: fatal signal %d at address %p (thread %ld)\n",
                   sig, si ? si->si_addr : nullptr, (long)gettid());
  if (n > 0) (void)!write(2, buf, (size_t)n);
  void* frames[64];
  int nf = backtrace(frames, 64);
  for (int i = 0; i < nf; ++i) {
    Dl_info info;
    if (dladdr(frames[i], &info) && info.dli_fname) {
      n = snprintf(buf, sizeof(buf), "  #%02d %s +0x%lx %s\n", i, info.dli_fname,
                   (unsigned long)((char*)frames[i] - (char*)info.dli_fbase),
                   info.dli_sname ? info.dli_sname : "");
    } else {
      n = snprintf(buf, sizeof(buf), "  #%02d %p\n", i, frames[i]);
    }
    if (n > 0) (void)!write(2, buf, (size_t)(n < (int)sizeof(buf) ? n : (int)sizeof(buf) - 1));
  }
  // restore the previous disposition and return: the faulting instruction
  // runs again and the previous handler (or the default action) takes over
  int s = slot_of(sig);
  if (s >= 0) sigaction(sig, &g_prev[s], nullptr);
}

}  // namespace

void install_crash_handler() {
  if (g_installed) return;
  backtrace(nullptr, 0);  // loads libgcc's unwinder outside the signal handler
  for (int i = 0; i < 4; ++i) {
    struct sigaction sa;
    std::memset(&sa, 0, sizeof(sa));
    sa.sa_sigaction = on_fatal;
    sa.sa_flags = SA_SIGINFO | SA_ONSTACK;
    sigemptyset(&sa.sa_mask);
    sigaction(kSignals[i], &sa, &g_prev[i]);
  }
  g_installed = 1;
}

void register_crash(py::module& m) {
  m.def("install_crash_handler", &install_crash_handler,
        "print native stacks on SIGSEGV/SIGBUS/SIGILL/SIGFPE, then defer to the previous handler");
}

}  // namespace rt
}  // namespace flodl
