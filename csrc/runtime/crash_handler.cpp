// crash_handler.cpp - print a native backtrace when the process dies on a
// fatal signal inside the runtime (SIGSEGV / SIGBUS / SIGFPE / SIGILL), then
// re-raise it with the default action so the exit status is unchanged.
// Installed once when the extension loads unless RAB_NO_CRASH_HANDLER is set.
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <initializer_list>
#include <cstring>

namespace rab {

namespace {

void on_fatal(int sig, siginfo_t* info, void*) {
  char head[160];
  const int n = snprintf(head, sizeof(head), "\n[rab] fatal signal %d (%s) at address %p; native backtrace:\n",
                         sig, strsignal(sig), info ? info->si_addr : nullptr);
  if (n > 0) (void)!write(2, head, static_cast<size_t>(n));
  void* frames[64];
  const int depth = backtrace(frames, 64);
  backtrace_symbols_fd(frames, depth, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}

}  // namespace

void install_crash_handler() {
  if (std::getenv("RAB_NO_CRASH_HANDLER") != nullptr) return;
  struct sigaction sa;
  std::memset(&sa, 0, sizeof(sa));
  sa.sa_sigaction = on_fatal;
  sa.sa_flags = SA_SIGINFO | SA_RESETHAND;
  sigemptyset(&sa.sa_mask);
  for (int sig : {SIGSEGV, SIGBUS, SIGFPE, SIGILL}) sigaction(sig, &sa, nullptr);
}

}  // namespace rab
