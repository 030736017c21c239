// TEST INFRASTRUCTURE: replays a text script of allocator / cache-manager /
// scheduler operations against the qwenvl_paged API and returns a trace of
// every return value and of the full bookkeeping state after each step.
//
// The same source is compiled twice: against this library's headers
// (tests/native/qvp_replay.cpp) and against the reference's own headers and
// sources (oracle/ref_replay.cpp, namespace renamed). Identical traces mean
// bit-identical ids, reference counts, generations, states, stats, swap slot
// ids, table entries and scheduler decisions.
//
// The includer defines REPLAY_MAKE_ALLOCATOR(config) to build its allocator.
//
// Script: one operation per line, whitespace separated.
//   init T L H D E blocks swap_slots [max_active max_tokens watermark]
//   create s | fork p c | reserve s n | write s pos | swapout s | swapin s
//   release s | view s | alloc | rel id | retain id | copy a b
//   bswapout id | bswapin slot | discard slot
//   failstore n | failload n        (the swap backend fails its nth next store / load)
//   enqueue r s prompt | schedule | complete r | cancel r | preempt r | resume r
#pragma once

#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/Scheduler.h"
#include "qwenvl_paged/SwapBackend.h"

#include <memory>
#include <set>
#include <sstream>
#include <string>
#include <vector>

namespace replay {

namespace qp = qwenvl_paged;

// Fault injection: a swap backend that forwards to another one but fails its
// Nth store or load from the moment it is armed (then behaves again).
class FailingSwapBackend final : public qp::SwapBackend {
public:
    explicit FailingSwapBackend(qp::SwapBackend& inner) : inner_(inner) {}
    std::optional<qp::SwapSlotId> store(const qp::PhysicalBlock& block) override {
        if (store_countdown_ > 0 && --store_countdown_ == 0) return std::nullopt;
        return inner_.store(block);
    }
    bool load(qp::SwapSlotId slot, qp::PhysicalBlock& block) override {
        if (load_countdown_ > 0 && --load_countdown_ == 0) return false;
        return inner_.load(slot, block);
    }
    void discard(qp::SwapSlotId slot) override { inner_.discard(slot); }
    std::size_t resident_slots() const noexcept override { return inner_.resident_slots(); }
    void fail_store(int nth) { store_countdown_ = nth; }
    void fail_load(int nth) { load_countdown_ = nth; }

private:
    qp::SwapBackend& inner_;
    int store_countdown_ = 0;
    int load_countdown_ = 0;
};

template <typename Opt>
std::string show(const Opt& o) {
    std::ostringstream s;
    if (o.has_value())
        s << *o;
    else
        s << "none";
    return s.str();
}

inline std::string run(const std::string& script) {
    std::istringstream in(script);
    std::ostringstream out;
    std::unique_ptr<qp::HostSwapBackend> swap;
    std::unique_ptr<FailingSwapBackend> faulty;
    std::unique_ptr<qp::MemoryAllocator> alloc;
    std::unique_ptr<qp::KVCacheManager> cache;
    std::unique_ptr<qp::Scheduler> sched;
    std::set<qp::SequenceId> seqs;
    std::set<qp::RequestId> reqs;
    std::string line;
    int n = 0;
    auto dump = [&]() {
        const qp::AllocatorStats st = alloc->stats();
        out << "  stats " << st.total_blocks << ' ' << st.free_blocks << ' ' << st.active_blocks << ' '
            << st.shared_blocks << ' ' << st.swapped_blocks << ' ' << st.bytes_reserved << '\n';
        out << "  blocks";
        for (qp::PhysicalBlockId i = 0; i < st.total_blocks; ++i) {
            const qp::PhysicalBlockInfo* in = alloc->info(i);
            out << ' ' << in->id << ':' << int(in->state) << ':' << in->ref_count << ':' << in->generation;
        }
        out << '\n';
        for (qp::SequenceId s : seqs) {
            out << "  seq " << s << ' ' << cache->contains(s);
            const auto v = cache->cache_view(s);
            if (v) {
                for (const qp::BlockTableEntry& e : v->block_table->entries())
                    out << ' ' << e.logical.index << '/' << e.logical.start_token << '/' << e.logical.token_count
                        << '/' << e.logical.sequence_id << ':' << e.physical_id << ':' << e.writable << ':'
                        << show(e.swap_slot);
            }
            out << '\n';
        }
        if (sched) {
            out << "  reqs active=" << sched->active_size();
            for (qp::RequestId r : reqs) {
                const auto s = sched->state(r);
                out << ' ' << r << ':' << (s ? int(*s) : -1);
                const auto info = sched->preemption_info(r);
                if (info) out << '[' << info->reason << '|' << info->swapped_blocks << ']';
            }
            out << '\n';
        }
    };
    while (std::getline(in, line)) {
        std::istringstream t(line);
        std::string op;
        if (!(t >> op)) continue;
        ++n;
        out << n << ' ' << line << " ->";
        if (op == "init") {
            qp::BlockShape sh;
            long long slots = -1;
            std::uint32_t blocks = 0;
            t >> sh.tokens_per_block >> sh.num_layers >> sh.num_kv_heads >> sh.head_dim >> sh.bytes_per_element >>
                blocks >> slots;
            qp::AllocatorConfig cfg;
            cfg.block_shape = sh;
            cfg.max_blocks = blocks;
            sched.reset();
            cache.reset();
            alloc.reset(REPLAY_MAKE_ALLOCATOR(cfg));
            swap.reset();
            faulty.reset();
            if (slots >= 0) {
                swap = std::make_unique<qp::HostSwapBackend>(static_cast<std::size_t>(slots));
                faulty = std::make_unique<FailingSwapBackend>(*swap);
                alloc->set_swap_backend(faulty.get());
            }
            cache = std::make_unique<qp::KVCacheManager>(*alloc);
            qp::SchedulerConfig sc;
            if (t >> sc.max_active_requests >> sc.max_batch_tokens >> sc.preemption_watermark_blocks)
                sched = std::make_unique<qp::Scheduler>(sc, *cache, *alloc);
            seqs.clear();
            reqs.clear();
            out << " ok\n";
        } else if (op == "create") {
            qp::SequenceId s;
            t >> s;
            seqs.insert(s);
            qp::SequenceMetadata m;
            m.sequence_id = s;
            m.request_id = s;
            out << ' ' << cache->create_sequence(m) << '\n';
        } else if (op == "fork") {
            qp::SequenceId p, c;
            t >> p >> c;
            seqs.insert(c);
            qp::SequenceMetadata m;
            m.sequence_id = c;
            m.request_id = p;
            out << ' ' << cache->fork_sequence(p, m) << '\n';
        } else if (op == "reserve") {
            qp::SequenceId s;
            std::uint32_t k;
            t >> s >> k;
            out << ' ' << cache->reserve_tokens(s, k) << '\n';
        } else if (op == "write") {
            qp::SequenceId s;
            qp::TokenPosition pos;
            t >> s >> pos;
            out << ' ' << show(cache->ensure_token_writable(s, pos)) << '\n';
        } else if (op == "swapout") {
            qp::SequenceId s;
            t >> s;
            out << ' ' << cache->swap_out_sequence(s) << '\n';
        } else if (op == "swapin") {
            qp::SequenceId s;
            t >> s;
            out << ' ' << cache->swap_in_sequence(s) << '\n';
        } else if (op == "release") {
            qp::SequenceId s;
            t >> s;
            cache->release_sequence(s);
            out << " done\n";
        } else if (op == "view") {
            qp::SequenceId s;
            t >> s;
            const auto v = cache->cache_view(s);
            out << ' ' << v.has_value();
            if (v) {
                out << " valid=" << v->valid() << " shape=" << v->layout.shape.byte_size() << " mapped=";
                for (qp::LogicalBlockIndex i = 0; i < v->block_table->size() + 1; ++i)
                {
                    // resolvable = what makes block_bytes non-null on a pool
                    // with storage (the bookkeeping-only pool has no bytes)
                    const auto id = v->block_table->lookup(i);
                    out << ((id && v->allocator->block(*id) != nullptr) ? '1' : '0');
                }
            }
            out << '\n';
        } else if (op == "alloc") {
            out << ' ' << show(alloc->allocate()) << '\n';
        } else if (op == "rel") {
            qp::PhysicalBlockId id;
            t >> id;
            alloc->release(id);
            out << " done\n";
        } else if (op == "retain") {
            qp::PhysicalBlockId id;
            t >> id;
            alloc->retain(id);
            out << " done\n";
        } else if (op == "copy") {
            qp::PhysicalBlockId a, b;
            t >> a >> b;
            alloc->copy_block(a, b);
            out << " done\n";
        } else if (op == "bswapout") {
            qp::PhysicalBlockId id;
            t >> id;
            out << ' ' << show(alloc->swap_out(id)) << '\n';
        } else if (op == "bswapin") {
            qp::SwapSlotId slot;
            t >> slot;
            out << ' ' << show(alloc->swap_in(slot)) << '\n';
        } else if (op == "discard") {
            qp::SwapSlotId slot;
            t >> slot;
            alloc->discard_swapped(slot);
            out << " done\n";
        } else if (op == "failstore" && faulty) {
            int k;
            t >> k;
            faulty->fail_store(k);
            out << " armed\n";
        } else if (op == "failload" && faulty) {
            int k;
            t >> k;
            faulty->fail_load(k);
            out << " armed\n";
        } else if (op == "enqueue" && sched) {
            qp::Request r;
            t >> r.request_id >> r.root_sequence_id >> r.prompt_tokens;
            reqs.insert(r.request_id);
            seqs.insert(r.root_sequence_id);
            sched->enqueue(r);
            out << " done\n";
        } else if (op == "schedule" && sched) {
            const qp::BatchPlan p = sched->schedule_next();
            out << " prefill";
            for (auto r : p.prefill_requests) out << ' ' << r;
            out << " decode";
            for (auto r : p.decode_requests) out << ' ' << r;
            out << " tokens " << p.scheduled_tokens << '\n';
        } else if (op == "complete" && sched) {
            qp::RequestId r;
            t >> r;
            sched->complete_step(r, 1);
            out << " done\n";
        } else if (op == "cancel" && sched) {
            qp::RequestId r;
            t >> r;
            sched->cancel(r);
            out << " done\n";
        } else if (op == "preempt" && sched) {
            qp::RequestId r;
            t >> r;
            out << ' ' << sched->preempt(r, "test") << '\n';
        } else if (op == "resume" && sched) {
            qp::RequestId r;
            t >> r;
            out << ' ' << sched->resume(r) << '\n';
        } else {
            out << " unknown\n";
            continue;
        }
        if (alloc) dump();
    }
    return out.str();
}

}  // namespace replay
