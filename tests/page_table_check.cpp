// Checks of the paged KV pool's page allocator (csrc/page_table.h), built and
// run by tests/test_page_table_cpu.py. Prints "ok" and exits 0 when every check
// holds; prints the failing check and exits 1 otherwise.
#include <cstdio>
#include <random>
#include <set>
#include <vector>

#include "page_table.h"

#define CHECK(c)                                                  \
    do {                                                          \
        if (!(c)) {                                               \
            std::printf("check failed at line %d: %s\n", __LINE__, #c); \
            return 1;                                             \
        }                                                         \
    } while (0)

int main() {
    using tie::PageTable;
    {   // growth by prefix, first-free order, bounds
        PageTable t(3, 100, 10);   // 7 pages per sequence, 10 physical pages
        CHECK(t.pages_per_seq() == 7 && t.free_pages() == 10 && t.scratch_page() == 10);
        CHECK(t.map(0, 1));
        CHECK(t.mapped_pages(0) == 1 && t.page(0, 0) == 0 && t.free_pages() == 9);
        CHECK(t.map(0, 16) && t.mapped_pages(0) == 1);      // still one page
        CHECK(t.map(0, 17) && t.mapped_pages(0) == 2 && t.page(0, 1) == 1);
        CHECK(t.map(1, 40) && t.mapped_pages(1) == 3);
        CHECK(t.page(1, 0) == 2 && t.page(1, 2) == 4 && t.free_pages() == 5);
        CHECK(!t.map(2, 101));                              // past the capacity
        CHECK(!t.map(2, 100));                              // 7 pages, 5 free: refused...
        CHECK(t.mapped_pages(2) == 0 && t.free_pages() == 5);   // ...with nothing changed
        CHECK(!t.map(3, 1) && !t.map(-1, 1) && !t.map(0, -1));
        const std::vector<int>& v = t.device_view();
        CHECK(v.size() == 21 && v[0] == 0 && v[1] == 1 && v[2] == 10 && v[7] == 2 && v[14] == 10);
        CHECK(!t.dirty());
    }
    {   // release and reuse
        PageTable t(2, 64, 4);
        CHECK(t.map(0, 64) && t.free_pages() == 0);
        CHECK(!t.map(1, 1));
        t.release(0);
        CHECK(t.free_pages() == 4 && t.mapped_pages(0) == 0 && t.page(0, 0) == -1 && t.dirty());
        CHECK(t.map(1, 33) && t.page(1, 0) == 0 && t.page(1, 1) == 1 && t.page(1, 2) == 2);
        t.release(5);                                        // out of range: no-op
        CHECK(t.free_pages() == 1);
    }
    {   // random map / release against a model of the allocation
        std::mt19937 rng(12345);
        const int S = 9, cap = 200, P = 40;
        PageTable t(S, cap, P);
        std::vector<int> len(S, 0);
        for (int it = 0; it < 20000; ++it) {
            const int s = (int)(rng() % S);
            if (rng() % 5 == 0) {
                t.release(s);
                len[s] = 0;
            } else {
                const int want = (int)(rng() % (cap + 1));
                const int need = (want + 15) / 16, have = t.mapped_pages(s);
                const bool fits = need <= have || need - have <= t.free_pages();
                CHECK(t.map(s, want) == fits);
                if (fits && want > len[s]) len[s] = want;
            }
            // every mapped page is distinct, free + mapped = P, mapped is a prefix
            std::set<int> seen;
            int mapped = 0;
            for (int q = 0; q < S; ++q) {
                CHECK(t.mapped_pages(q) >= (len[q] + 15) / 16);
                for (int p = 0; p < t.pages_per_seq(); ++p) {
                    const int g = t.page(q, p);
                    CHECK((p < t.mapped_pages(q)) == (g >= 0));
                    if (g >= 0) {
                        CHECK(g < P && seen.insert(g).second);
                        ++mapped;
                    }
                }
            }
            CHECK(mapped + t.free_pages() == P);
        }
    }
    std::printf("ok\n");
    return 0;
}
