// ref_layout_shim.cpp — exports the reference's own stripe-map header as C symbols.
//
// TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile (target `ref`) against
// common/kv_layout.h where it lies in the reference tree (-I<reference>/common),
// into oracle/_ref/libkv_layout_ref.so. The tests use it to pin the C
// restatement's ko_node_of / ko_seg_row / offsets against the reference's code.
#include <cstdint>

#include "kv_layout.h"

extern "C" {
uint32_t ref_per_layer_seg_rows(uint32_t layer_rows, uint32_t node_num)
{
    return KvLayoutPerLayerSegRows(layer_rows, node_num);
}

uint32_t ref_node_of(uint32_t row, uint32_t stripe, uint32_t node_num)
{
    KvLayout lay{node_num, 1, 1, 1, 128, stripe};
    return KvLayoutNode(row, &lay);
}

uint32_t ref_seg_row_of(uint32_t row, uint32_t stripe, uint32_t node_num)
{
    KvLayout lay{node_num, 1, 1, 1, 128, stripe};
    return KvLayoutSegRow(row, &lay);
}

uint64_t ref_seg_offset(uint32_t layer, uint32_t row, uint32_t stripe, uint32_t node_num, uint32_t plsr,
                        uint32_t row_bytes)
{
    KvLayout lay{node_num, 1, 1, plsr, row_bytes, stripe};
    return KvLayoutSegOffset(layer, row, &lay);
}

int ref_validate(uint32_t node_num, uint32_t layer_num, uint32_t layer_rows, uint32_t plsr, uint32_t row_bytes,
                 uint32_t stripe)
{
    KvLayout lay{node_num, layer_num, layer_rows, plsr, row_bytes, stripe};
    return KvLayoutValidate(&lay);
}
}
