// tg_rcm_order: reverse Cuthill-McKee ordering of a square sparse matrix (host code).
//
// No counterpart in the reference: an optional preprocessing pass that renumbers rows and
// columns together so that rows which share columns get nearby numbers.  Applied as
// A' = P A P^T (and B' = P B for SpMM), it shortens the distance, in processing order,
// between the uses of each gathered dense row, which raises the L2 hit rate of the x / B
// / V gathers.  It does nothing for a pattern without such structure (uniformly random
// columns have none to find); it restores locality that a scrambled numbering hid.
//
// Cuthill-McKee: breadth-first search of the symmetrised pattern (A + A^T without the
// diagonal) from a pseudo-peripheral node (George and Liu's repeated-BFS heuristic: start
// at a node of minimum degree, move to a minimum-degree node of the last BFS level while
// the eccentricity grows), visiting each node's unvisited neighbours in increasing
// degree; each connected component in turn, components started from their
// minimum-degree node; the final order is reversed.
#include <algorithm>
#include <cstring>
#include <vector>

#include "tg_common.cuh"

namespace {

struct Graph {
    std::vector<int64_t> ptr;
    std::vector<int64_t> adj;
    std::vector<int64_t> deg;
};

// A + A^T without self loops, duplicates removed, neighbour lists sorted.
Graph symmetrise(int64_t n, const int64_t* indptr, const int64_t* indices) {
    Graph g;
    std::vector<int64_t> cnt(n + 1, 0);
    for (int64_t i = 0; i < n; ++i)
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
            const int64_t j = indices[p];
            if (j == i) continue;
            ++cnt[i + 1];
            ++cnt[j + 1];
        }
    for (int64_t i = 0; i < n; ++i) cnt[i + 1] += cnt[i];
    std::vector<int64_t> adj(cnt[n]);
    std::vector<int64_t> fill(cnt.begin(), cnt.end() - 1);
    for (int64_t i = 0; i < n; ++i)
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
            const int64_t j = indices[p];
            if (j == i) continue;
            adj[fill[i]++] = j;
            adj[fill[j]++] = i;
        }
    // sort each list and drop duplicates, compacting the lists to the front in place
    // (the write position never passes the read position)
    g.ptr.assign(n + 1, 0);
    g.deg.assign(n, 0);
    int64_t w = 0;
    for (int64_t i = 0; i < n; ++i) {
        std::sort(adj.begin() + cnt[i], adj.begin() + cnt[i + 1]);
        g.ptr[i] = w;
        int64_t prev = -1;
        for (int64_t r = cnt[i]; r < cnt[i + 1]; ++r) {
            const int64_t v = adj[r];
            if (v != prev) adj[w++] = v;
            prev = v;
        }
        g.deg[i] = w - g.ptr[i];
    }
    g.ptr[n] = w;
    adj.resize(w);
    g.adj.swap(adj);
    return g;
}

// BFS levels from `root` over nodes not yet ordered; fills `last` with the nodes of the
// last level and returns the number of levels.  `level` is -1 everywhere on entry and on
// return (only the nodes this search reached are touched).
int64_t bfs_last_level(const Graph& g, int64_t root, std::vector<int64_t>& level, std::vector<int64_t>& queue,
                       std::vector<int64_t>& last, const std::vector<char>& done) {
    queue.clear();
    queue.push_back(root);
    level[root] = 0;
    int64_t maxl = 0;
    for (size_t h = 0; h < queue.size(); ++h) {
        const int64_t u = queue[h];
        for (int64_t p = g.ptr[u]; p < g.ptr[u + 1]; ++p) {
            const int64_t v = g.adj[p];
            if (done[v] || level[v] >= 0) continue;
            level[v] = level[u] + 1;
            maxl = std::max(maxl, level[v]);
            queue.push_back(v);
        }
    }
    last.clear();
    for (int64_t u : queue) {
        if (level[u] == maxl) last.push_back(u);
        level[u] = -1;
    }
    return maxl + 1;
}

}  // namespace

using namespace tg;

extern "C" int tg_rcm_order(int64_t n, const int64_t* indptr, const int64_t* indices, int64_t* perm) {
    if (n < 0) return set_error(TG_EINVAL, "tg_rcm_order: negative size");
    if (n == 0) return TG_OK;
    if (!indptr || !perm || (indptr[n] > 0 && !indices)) return set_error(TG_EINVAL, "tg_rcm_order: null argument");
    for (int64_t i = 0; i < n; ++i)
        if (indptr[i + 1] < indptr[i]) return set_error(TG_EINVAL, "tg_rcm_order: indptr decreasing at row %lld",
                                                        (long long)i);
    for (int64_t p = 0; p < indptr[n]; ++p)
        if (indices[p] < 0 || indices[p] >= n)
            return set_error(TG_EBOUNDS, "tg_rcm_order: column index out of range at %lld", (long long)p);
    const Graph g = symmetrise(n, indptr, indices);
    // component starts are tried in increasing degree (ties: lower index)
    std::vector<int64_t> by_deg(n);
    for (int64_t i = 0; i < n; ++i) by_deg[i] = i;
    std::stable_sort(by_deg.begin(), by_deg.end(), [&](int64_t a, int64_t b) { return g.deg[a] < g.deg[b]; });
    std::vector<char> done(n, 0);
    std::vector<int64_t> order;
    order.reserve(n);
    std::vector<int64_t> level(n, -1), queue, last, nbr;
    queue.reserve(n);
    for (int64_t s : by_deg) {
        if (done[s]) continue;
        // pseudo-peripheral start within s's component
        int64_t root = s;
        int64_t ecc = bfs_last_level(g, root, level, queue, last, done);
        for (int round = 0; round < 8; ++round) {
            int64_t cand = last[0];
            for (int64_t u : last)
                if (g.deg[u] < g.deg[cand] || (g.deg[u] == g.deg[cand] && u < cand)) cand = u;
            const int64_t e2 = bfs_last_level(g, cand, level, queue, last, done);
            if (e2 <= ecc) break;
            root = cand;
            ecc = e2;
        }
        // Cuthill-McKee from root
        const size_t first = order.size();
        order.push_back(root);
        done[root] = 1;
        for (size_t h = first; h < order.size(); ++h) {
            const int64_t u = order[h];
            nbr.clear();
            for (int64_t p = g.ptr[u]; p < g.ptr[u + 1]; ++p)
                if (!done[g.adj[p]]) {
                    done[g.adj[p]] = 1;
                    nbr.push_back(g.adj[p]);
                }
            std::sort(nbr.begin(), nbr.end(), [&](int64_t a, int64_t b) {
                return g.deg[a] != g.deg[b] ? g.deg[a] < g.deg[b] : a < b;
            });
            order.insert(order.end(), nbr.begin(), nbr.end());
        }
    }
    for (int64_t k = 0; k < n; ++k) perm[k] = order[n - 1 - k];
    return TG_OK;
}
