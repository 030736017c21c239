// TEST INFRASTRUCTURE: runner for test files built on gtest_shim/gtest/gtest.h.
// Every case runs in a forked child (one minute at most), so a case that
// crashes or hangs fails alone. Prints one line per case:
//   PASS <suite>.<name> | FAIL <suite>.<name> | CRASH <suite>.<name> signal N
// followed by the failure text, and exits 0 only when every case passed.
// With arguments, runs only the cases named <suite>.<name>.
#include <gtest/gtest.h>

#include <sys/wait.h>
#include <unistd.h>

#include <cstdio>
#include <string>

namespace {

// Child side: runs the case, writes "<failed>\n<log>" to `fd`.
[[noreturn]] void run_child(const testing::internal::Case& c, int fd) {
    alarm(60);
    testing::Test* t = c.make();
    t->SetUp();
    if (!testing::internal::state().fatal) t->TestBody();
    t->TearDown();
    delete t;
    const testing::internal::State& s = testing::internal::state();
    const std::string msg = std::string(s.failed ? "1\n" : "0\n") + s.log;
    std::size_t off = 0;
    while (off < msg.size()) {
        const ssize_t n = write(fd, msg.data() + off, msg.size() - off);
        if (n <= 0) break;
        off += static_cast<std::size_t>(n);
    }
    close(fd);
    _exit(s.failed ? 1 : 0);
}

}  // namespace

int main(int argc, char** argv) {
    int failures = 0, run = 0;
    for (const testing::internal::Case& c : testing::internal::cases()) {
        const std::string full = c.suite + "." + c.name;
        if (argc > 1) {
            bool wanted = false;
            for (int i = 1; i < argc; ++i) wanted = wanted || full == argv[i];
            if (!wanted) continue;
        }
        ++run;
        int fds[2];
        if (pipe(fds) != 0) return 2;
        std::fflush(stdout);
        const pid_t pid = fork();
        if (pid == 0) {
            close(fds[0]);
            run_child(c, fds[1]);
        }
        close(fds[1]);
        std::string out;
        char buf[4096];
        ssize_t n;
        while ((n = read(fds[0], buf, sizeof(buf))) > 0) out.append(buf, static_cast<std::size_t>(n));
        close(fds[0]);
        int status = 0;
        waitpid(pid, &status, 0);
        if (WIFSIGNALED(status)) {
            std::printf("CRASH %s signal %d\n", full.c_str(), WTERMSIG(status));
            ++failures;
        } else if (out.empty() || out[0] != '0' || WEXITSTATUS(status) != 0) {
            std::printf("FAIL %s\n%s", full.c_str(), out.size() > 2 ? out.c_str() + 2 : "");
            ++failures;
        } else {
            std::printf("PASS %s\n", full.c_str());
        }
    }
    std::printf("%d cases, %d failed\n", run, failures);
    return failures == 0 ? 0 : 1;
}
