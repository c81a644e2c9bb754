/* Minimal ggml stand-in for the XQ_B200 backend self-tests: the functions the
 * backend calls from libggml-base (buffer init, backend registration, graph
 * node access, ggml_nbytes), over the layouts of ggml_abi_mirror.h.  The
 * graph here is a plain node list; the real ggml_cgraph differs and is only
 * ever touched through these accessors. */
#include <stdlib.h>
#include <string.h>

#include "ggml_abi_mirror.h"

struct ggml_cgraph {
    int n_nodes;
    struct ggml_tensor **nodes;
};

static ggml_backend_reg_t g_regs[16];
static int g_nregs;

ggml_backend_buffer_t ggml_backend_buffer_init(ggml_backend_buffer_type_t buft,
                                               struct ggml_backend_buffer_i iface, void *context,
                                               size_t size) {
    ggml_backend_buffer_t b = (ggml_backend_buffer_t)calloc(1, sizeof(*b));
    b->iface = iface;
    b->buft = buft;
    b->context = context;
    b->size = size;
    b->usage = GGML_BACKEND_BUFFER_USAGE_ANY;
    return b;
}

void ggml_backend_register(ggml_backend_reg_t reg) {
    if (g_nregs < 16)
        g_regs[g_nregs++] = reg;
}

int ggml_graph_n_nodes(struct ggml_cgraph *g) { return g->n_nodes; }

struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *g, int i) {
    return g->nodes[i < 0 ? g->n_nodes + i : i];
}

static size_t type_size(int t) { return t == 0 ? 4 : t == 1 ? 2 : t == 8 ? 34 : 18; }
static int blck(int t) { return (t == 0 || t == 1) ? 1 : 32; }

size_t ggml_nbytes(const struct ggml_tensor *t) {
    size_t n = type_size(t->type);
    n = (size_t)(t->ne[0] / blck(t->type)) * n;
    for (int i = 1; i < 4; ++i)
        if (t->ne[i] > 1)
            n += (size_t)(t->ne[i] - 1) * t->nb[i];
    return n;
}

/* test helpers */
int xq_mock_registered(void) { return g_nregs; }
ggml_backend_reg_t xq_mock_reg(int i) { return i < g_nregs ? g_regs[i] : 0; }
void xq_mock_buffer_free(ggml_backend_buffer_t b) {
    b->iface.free_buffer(b);
    free(b);
}
